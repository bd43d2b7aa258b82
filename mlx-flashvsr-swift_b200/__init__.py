"""B200-native LCSA hot path of FlashVSR — the host-side mirror of the reference's operator interface.

The reference (xocialize/mlx-flashvsr-swift) exposes the path as Swift functions on MLXArrays:
    draftBlockMaskAndProbs(qW:kW:heads:qSlices:spatialBlocks:local:topk:)   Sources/FlashVSRMLX/DiT.swift:158-174
    kernelBlockAttention(q:k:v:blockMask:heads:simdgroups:)                 Sources/FlashVSRMLX/SparseAttention.swift:169-187
    FlashVSRAttentionOps.kernel(q:k:v:blockMask:heads:)                     Sources/FlashVSRMLX/SparseAttention.swift:190-201
    the window K/V cache of blockForward                                    Sources/FlashVSRMLX/DiT.swift:507-511, 532-538
This module offers the same operations, with the same argument meaning, on CUDA torch tensors, by calling the C ABI of
``include/fvsr_lcsa.h`` (``libfvsr_lcsa.so``, hand-written sm_100a kernels) through ctypes. torch is used only for
device memory and the current stream. There is no fallback: if the library is missing, importing this package fails.
Of FlashVSRAttentionOps only the `kernel` lane is offered; the reference's `dense` and `gathered` study lanes are
probe code, not part of this path.

Where the reference traps on a bad shape (``precondition``), these functions raise ``FVSRError`` carrying the C
status and message.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = PKG_DIR / "libfvsr_lcsa.so"

FVSR_OK, FVSR_EINVAL, FVSR_ECUDA, FVSR_ETIMEOUT, FVSR_ENOMEM, FVSR_EUNSUPPORTED = range(6)
FVSR_F32, FVSR_BF16 = 0, 1
FVSR_LINEAR, FVSR_LINEAR_GELU, FVSR_LINEAR_GATED_RESIDUAL = 0, 1, 2

EXPORTED = [
    "fvsr_version", "fvsr_status_string", "fvsr_last_error", "fvsr_device_check", "fvsr_wait_probe",
    "fvsr_lcsa_workspace_size",
    "fvsr_lcsa_pool", "fvsr_lcsa_select", "fvsr_lcsa_attention", "fvsr_lcsa_layer", "fvsr_lcsa_attention_mask",
    "fvsr_kv_cache_create",
    "fvsr_kv_cache_destroy", "fvsr_kv_cache_reset", "fvsr_kv_cache_slices", "fvsr_kv_cache_append",
    "fvsr_kv_cache_trim", "fvsr_kv_cache_gather", "fvsr_kv_cache_state", "fvsr_lcsa_forward",
    "fvsr_lcsa_select_noalloc", "fvsr_lcsa_attention_range", "fvsr_lcsa_item_order", "fvsr_lcsa_schedule_size",
    "fvsr_lcsa_schedule", "fvsr_lcsa_attention_scheduled", "fvsr_lcsa_prepare", "fvsr_lcsa_forward_tokens",
    "fvsr_stream_chunk_geometry", "fvsr_stream_create", "fvsr_stream_destroy", "fvsr_stream_begin",
    "fvsr_stream_workspace_size", "fvsr_stream_start_chunk", "fvsr_stream_rope", "fvsr_stream_layer",
    "fvsr_kv_cache_create_padded", "fvsr_kv_cache_reserve", "fvsr_kv_cache_commit", "fvsr_lcsa_forward_shard",
    "fvsr_lcsa_partial_size", "fvsr_lcsa_select_shard", "fvsr_lcsa_attend_shard", "fvsr_linear", "fvsr_linear_qkv",
    "fvsr_layernorm", "fvsr_rmsnorm", "fvsr_cross_attention",
]


class Params(ctypes.Structure):
    """struct fvsr_lcsa_params."""
    _fields_ = [(n, ctypes.c_int32) for n in
                ("heads", "head_dim", "bh", "bw", "q_slices", "kv_slices", "local_range", "topk", "dtype")]


class FVSRError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"fvsr status {status}: {message}")
        self.status = status


_lib = None


def build(force: bool = False) -> Path:
    """Compile libfvsr_lcsa.so in-tree (nvcc, sm_100a)."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("fvsr_b200_build", PKG_DIR / "build.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.build(force=force)


def lib() -> ctypes.CDLL:
    """The loaded C ABI. Raises if the library has not been built — the CUDA path is the only path."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ImportError(f"{LIB_PATH} is not built; run build() (nvcc, sm_100a) first")
    L = ctypes.CDLL(str(LIB_PATH))
    P, I32, I64, SZ = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t
    PP = ctypes.POINTER(Params)
    sigs = {
        "fvsr_version": ([], I32),
        "fvsr_status_string": ([ctypes.c_int], ctypes.c_char_p),
        "fvsr_last_error": ([], ctypes.c_char_p),
        "fvsr_device_check": ([P], ctypes.c_int),
        "fvsr_wait_probe": ([ctypes.c_uint32, P], ctypes.c_int),
        "fvsr_lcsa_workspace_size": ([PP, ctypes.POINTER(SZ)], ctypes.c_int),
        "fvsr_lcsa_pool": ([PP, P, I64, P, P], ctypes.c_int),
        "fvsr_lcsa_select": ([PP, P, P, P, P, P, P, P, P, SZ, P], ctypes.c_int),
        "fvsr_lcsa_attention": ([PP, P, P, P, P, P, P, P], ctypes.c_int),
        "fvsr_lcsa_layer": ([PP, P, P, P, P, P, P, P, SZ, P], ctypes.c_int),
        "fvsr_lcsa_attention_mask": ([PP, P, P, P, P, P, P, SZ, P], ctypes.c_int),
        "fvsr_kv_cache_create": ([PP, I32, I32, ctypes.POINTER(P)], ctypes.c_int),
        "fvsr_kv_cache_destroy": ([P], ctypes.c_int),
        "fvsr_kv_cache_reset": ([P], ctypes.c_int),
        "fvsr_kv_cache_slices": ([P, ctypes.POINTER(I32)], ctypes.c_int),
        "fvsr_kv_cache_append": ([P, P, P, I32, P], ctypes.c_int),
        "fvsr_kv_cache_trim": ([P], ctypes.c_int),
        "fvsr_kv_cache_gather": ([P, P, P, P], ctypes.c_int),
        "fvsr_kv_cache_state": ([P, P, ctypes.POINTER(I32)], ctypes.c_int),
        "fvsr_lcsa_forward": ([PP, P, P, P, P, P, P, P, P, SZ, P], ctypes.c_int),
        "fvsr_lcsa_select_noalloc": ([PP, P, P, P, P, P, P, P, P], ctypes.c_int),
        "fvsr_lcsa_attention_range": ([PP, P, P, P, P, P, P, I32, I32, P, P], ctypes.c_int),
        "fvsr_lcsa_item_order": ([PP, P, I32, I32, P, P], ctypes.c_int),
        "fvsr_lcsa_schedule_size": ([PP, I32, ctypes.POINTER(SZ)], ctypes.c_int),
        "fvsr_lcsa_schedule": ([PP, P, I32, I32, P, SZ, P], ctypes.c_int),
        "fvsr_lcsa_attention_scheduled": ([PP, P, P, P, P, P, P, I32, I32, P, SZ, P], ctypes.c_int),
        "fvsr_lcsa_prepare": ([PP, P, P, P, P, P, ctypes.c_float, P, P, P, P, P, P, P, P], ctypes.c_int),
        "fvsr_lcsa_forward_tokens": ([PP, P, P, P, P, P, ctypes.c_float, P, P, P, P, P, P, P, P, SZ, P],
                                     ctypes.c_int),
        "fvsr_stream_chunk_geometry": ([I32, I32, I32, I32, ctypes.c_double, I32, I32, PP, ctypes.POINTER(I32),
                                        ctypes.POINTER(I32)], ctypes.c_int),
        "fvsr_stream_create": ([I32, I32, I32, I32, I32, ctypes.c_double, ctypes.c_double, I32, ctypes.POINTER(P)],
                               ctypes.c_int),
        "fvsr_stream_destroy": ([P], ctypes.c_int),
        "fvsr_stream_begin": ([P], ctypes.c_int),
        "fvsr_stream_workspace_size": ([P, ctypes.POINTER(SZ)], ctypes.c_int),
        "fvsr_stream_start_chunk": ([P, I32, P], ctypes.c_int),
        "fvsr_stream_rope": ([P, ctypes.POINTER(P), ctypes.POINTER(P), ctypes.POINTER(I64)], ctypes.c_int),
        "fvsr_stream_layer": ([P, I32, P, P, P, P, P, ctypes.c_float, P, P, P, P, P, SZ, P], ctypes.c_int),
        "fvsr_kv_cache_create_padded": ([PP, I32, I32, I32, ctypes.POINTER(P)], ctypes.c_int),
        "fvsr_kv_cache_reserve": ([P, ctypes.POINTER(P), ctypes.POINTER(P), ctypes.POINTER(P)], ctypes.c_int),
        "fvsr_kv_cache_commit": ([P], ctypes.c_int),
        "fvsr_lcsa_forward_shard": ([PP, P, I32, I32, P, P, P, P, P, P, P, SZ, P], ctypes.c_int),
        "fvsr_lcsa_partial_size": ([PP, I32, I32, ctypes.POINTER(SZ)], ctypes.c_int),
        "fvsr_lcsa_select_shard": ([PP, P, I32, I32, P, P, P, P, SZ, I32, P], ctypes.c_int),
        "fvsr_lcsa_attend_shard": ([PP, P, I32, I32, P, P, P, SZ, P, P, P, P, SZ, P], ctypes.c_int),
        "fvsr_linear": ([I32, I32, I32, P, P, P, I32, P, P, P, P], ctypes.c_int),
        "fvsr_linear_qkv": ([I32, I32, I32, P, P, P, P, P, P, P], ctypes.c_int),
        "fvsr_layernorm": ([I32, I32, P, P, P, P, P, ctypes.c_float, P, P], ctypes.c_int),
        "fvsr_rmsnorm": ([I32, I32, P, P, ctypes.c_float, P, P], ctypes.c_int),
        "fvsr_cross_attention": ([I32, I32, I32, P, P, P, P, P], ctypes.c_int),
    }
    for name, (args, res) in sigs.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res
    _lib = L
    return L


def _check(status: int) -> None:
    if status != FVSR_OK:
        raise FVSRError(status, lib().fvsr_last_error().decode())


# ---------------------------------------------------------------------------------------------------------------
# Geometry (DiT.swift:473-485)
# ---------------------------------------------------------------------------------------------------------------

@dataclass
class Geometry:
    """One LCSA call's geometry: ``s = bh·bw`` spatial blocks per temporal slice, ``Nq = q_slices·s`` query blocks,
    ``Nk = kv_slices·s`` key blocks (cache ⊕ current), locality range R and the integer top-k."""
    heads: int
    bh: int
    bw: int
    q_slices: int
    kv_slices: int
    local_range: int = 11
    topk: int = 0
    dtype: int = FVSR_BF16

    @property
    def s(self) -> int:
        return self.bh * self.bw

    @property
    def nq(self) -> int:
        return self.q_slices * self.s

    @property
    def nk(self) -> int:
        return self.kv_slices * self.s

    @property
    def channels(self) -> int:
        return self.heads * 128

    def params(self) -> Params:
        return Params(self.heads, 128, self.bh, self.bw, self.q_slices, self.kv_slices, self.local_range, self.topk,
                      self.dtype)

    def allowed_per_row(self) -> int:
        """Locality-allowed (query block, key block) pairs in one (head, slice) selection row."""
        half = self.local_range // 2
        tot = 0
        for qr in range(self.bh):
            nr = sum(1 for kr in range(self.bh) if qr - half <= kr <= qr - half + self.local_range - 1)
            for qc in range(self.bw):
                nc = sum(1 for kc in range(self.bw) if qc - half <= kc <= qc - half + self.local_range - 1)
                tot += nr * nc
        return tot * self.kv_slices

    @staticmethod
    def topk_from_ratio(s: int, ratio: float) -> int:
        """DiT.swift:482: topk = Int(Double(s·s)·topkRatio) − 1."""
        return int(float(s * s) * ratio) - 1


def _torch():
    import torch
    return torch


def _dtype_code(t) -> int:
    torch = _torch()
    if t.dtype == torch.bfloat16:
        return FVSR_BF16
    if t.dtype == torch.float32:
        return FVSR_F32
    raise FVSRError(FVSR_EINVAL, f"tensors must be bfloat16 or float32, got {t.dtype}")


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(stream=None):
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def _rows(t):
    """(1, L, C) or (L, C) → (L, C) view (the reference's batch-1 contract, SparseAttention.swift:173)."""
    if t.dim() == 3:
        if t.shape[0] != 1:
            raise FVSRError(FVSR_EINVAL, "batch must be 1")
        t = t[0]
    if not t.is_cuda or not t.is_contiguous():
        raise FVSRError(FVSR_EINVAL, "tensors must be contiguous CUDA tensors")
    return t


def workspace_size(geom: Geometry) -> int:
    n = ctypes.c_size_t(0)
    p = geom.params()
    _check(lib().fvsr_lcsa_workspace_size(ctypes.byref(p), ctypes.byref(n)))
    return int(n.value)


def make_workspace(geom: Geometry, device=None):
    torch = _torch()
    return torch.empty(workspace_size(geom), dtype=torch.uint8, device=device or "cuda")


def pool(x, geom: Geometry, out=None, stream=None):
    """fp32 block means (DiT.swift:161-162): x (N·128, H·128) → (N, H·128) fp32."""
    torch = _torch()
    x = _rows(x)
    nblocks = x.shape[0] // 128
    if out is None:
        out = torch.empty((nblocks, x.shape[1]), dtype=torch.float32, device=x.device)
    g = Geometry(**{**geom.__dict__, "dtype": _dtype_code(x)})
    p = g.params()
    _check(lib().fvsr_lcsa_pool(ctypes.byref(p), _ptr(x), nblocks, _ptr(out), _stream(stream)))
    return out


def draft_block_mask_and_probs(qW, kW, geom: Geometry, pooled_k=None, want_mask: bool = True,
                               want_probs: bool = True, workspace=None, stream=None):
    """draftBlockMaskAndProbs (DiT.swift:158-174). qW (Nq·128, H·128), kW (Nk·128, H·128) window order.
    Returns dict(mask (H,Nq,Nk) uint8, probs (H,Nq,Nk) f32, kidx (H,Nq,Nk) i32 kept-first ascending, kcnt (H,Nq))."""
    torch = _torch()
    q = _rows(qW)
    k = None if kW is None else _rows(kW)
    g = Geometry(**{**geom.__dict__, "dtype": _dtype_code(q)})
    dev = q.device
    kidx = torch.empty((g.heads, g.nq, g.nk), dtype=torch.int32, device=dev)
    kcnt = torch.empty((g.heads, g.nq), dtype=torch.int32, device=dev)
    mask = torch.empty((g.heads, g.nq, g.nk), dtype=torch.uint8, device=dev) if want_mask else None
    probs = torch.empty((g.heads, g.nq, g.nk), dtype=torch.float32, device=dev) if want_probs else None
    ws = workspace if workspace is not None else make_workspace(g, dev)
    p = g.params()
    _check(lib().fvsr_lcsa_select(ctypes.byref(p), _ptr(q), _ptr(k), _ptr(pooled_k), _ptr(kidx), _ptr(kcnt),
                                  _ptr(mask), _ptr(probs), _ptr(ws), ws.numel(), _stream(stream)))
    return {"mask": mask, "probs": probs, "kidx": kidx, "kcnt": kcnt}


def block_sparse_attention(q, k, v, kidx, kcnt, geom: Geometry, out=None, stream=None):
    """Attention over the kept blocks given index lists. q (Nq·128, H·128), k / v (Nk·128, H·128)."""
    torch = _torch()
    shape = q.shape
    q2, k2, v2 = _rows(q), _rows(k), _rows(v)
    g = Geometry(**{**geom.__dict__, "dtype": _dtype_code(q2)})
    if out is None:
        out = torch.empty_like(q2)
    p = g.params()
    _check(lib().fvsr_lcsa_attention(ctypes.byref(p), _ptr(q2), _ptr(k2), _ptr(v2), _ptr(kidx), _ptr(kcnt),
                                     _ptr(out), _stream(stream)))
    return out.reshape(shape)


def lcsa_layer(q, k, v, geom: Geometry, out=None, kidx=None, kcnt=None, workspace=None, stream=None):
    """One layer without a cache (DiT.swift:512-527): draftBlockMaskAndProbs then kernelBlockAttention in one call —
    pooling, the selection (which also orders the items longest first) and the attention. q (Nq·128, H·128), k / v
    (Nk·128, H·128) window order; returns out like q."""
    torch = _torch()
    shape = q.shape
    q2, k2, v2 = _rows(q), _rows(k), _rows(v)
    g = Geometry(**{**geom.__dict__, "dtype": _dtype_code(q2)})
    if out is None:
        out = torch.empty_like(q2)
    ws = workspace if workspace is not None else make_workspace(g, q2.device)
    p = g.params()
    _check(lib().fvsr_lcsa_layer(ctypes.byref(p), _ptr(q2), _ptr(k2), _ptr(v2), _ptr(_rows(out)), _ptr(kidx),
                                 _ptr(kcnt), _ptr(ws), ws.numel(), _stream(stream)))
    return out.reshape(shape)


def item_order(kcnt, geom: Geometry, item_begin: int, item_count: int, order=None, stream=None):
    """Longest-first order of the items [item_begin, item_begin + item_count): the non-empty items of each head in
    turn by decreasing kcnt (ties by id), then the range's empty items by id."""
    torch = _torch()
    if order is None:
        order = torch.empty(item_count, dtype=torch.int32, device=kcnt.device)
    p = geom.params()
    _check(lib().fvsr_lcsa_item_order(ctypes.byref(p), _ptr(kcnt), int(item_begin), int(item_count), _ptr(order),
                                      _stream(stream)))
    return order


def block_sparse_attention_range(q, k, v, kidx, kcnt, geom: Geometry, item_begin: int, item_count: int, out,
                                 order=None, stream=None):
    """block_sparse_attention for work items [item_begin, item_begin + item_count) only (item = h·Nq + qb), in the
    given order (from item_order) or ascending."""
    q2, k2, v2, o2 = _rows(q), _rows(k), _rows(v), _rows(out)
    g = Geometry(**{**geom.__dict__, "dtype": _dtype_code(q2)})
    p = g.params()
    _check(lib().fvsr_lcsa_attention_range(ctypes.byref(p), _ptr(q2), _ptr(k2), _ptr(v2), _ptr(kidx), _ptr(kcnt),
                                           _ptr(o2), int(item_begin), int(item_count), _ptr(order), _stream(stream)))
    return out


def schedule_size(geom: Geometry, item_count: int) -> int:
    """Bytes of the device buffer fvsr_lcsa_schedule fills for a range of item_count items (current device)."""
    n = ctypes.c_size_t(0)
    p = geom.params()
    _check(lib().fvsr_lcsa_schedule_size(ctypes.byref(p), int(item_count), ctypes.byref(n)))
    return n.value


def schedule_is_persistent(geom: Geometry, item_begin: int, item_count: int, sms: int) -> bool:
    """Whether make_schedule gives the range the persistent partition (the C library's rule: a bf16 range inside one
    head with at most 8 items per SM); otherwise it gets the longest-first order of the per-item kernel."""
    if item_count <= 0 or geom.dtype != FVSR_BF16:
        return False
    hr = min(geom.heads, (item_count - 1) // geom.nq + 2)
    room = item_count <= 8 * sms and item_count <= 4096 and hr <= 63 and sms * hr <= 16384
    return room and item_begin // geom.nq == (item_begin + item_count - 1) // geom.nq


def make_schedule(kcnt, geom: Geometry, item_begin: int, item_count: int, buf=None, stream=None):
    """Work schedule of the items [item_begin, item_begin + item_count): for a short range (at most 8 items per SM)
    the persistent kernel's partition — per head, the head's kept key blocks in equal shares per SM, cut items merged
    afterwards — else the longest-first item order. Returns the uint8 device buffer (reused by
    block_sparse_attention_scheduled)."""
    torch = _torch()
    nbytes = schedule_size(geom, item_count)
    if buf is None:
        buf = torch.empty(nbytes, dtype=torch.uint8, device=kcnt.device)
    p = geom.params()
    _check(lib().fvsr_lcsa_schedule(ctypes.byref(p), _ptr(kcnt), int(item_begin), int(item_count), _ptr(buf),
                                    buf.numel(), _stream(stream)))
    return buf


def schedule_view(buf, geom: Geometry, item_count: int):
    """Host view of a persistent-mode schedule buffer (synchronises): header (segments, cut items, pieces, heads of
    the range, empty items), per-SM segment ranges, segments (item, first list position, length, piece slot or -1),
    merge records (item, first slot, pieces) and the empty items."""
    import numpy as np
    torch = _torch()
    torch.cuda.synchronize(buf.device)
    b = buf.cpu().numpy()
    a = lambda x: (x + 255) & ~255
    G = torch.cuda.get_device_properties(buf.device).multi_processor_count
    hr = min(geom.heads, (item_count - 1) // geom.nq + 2)
    off_seg_begin = a(32) + a(item_count * 4)
    off_segs = off_seg_begin + a((G + 1) * 4)
    off_comb = off_segs + a((item_count + G * hr) * 16)
    off_empties = off_comb + a(G * hr * 16)
    hdr = b[:20].view(np.int32)
    n_segs, n_comb, n_empty = int(hdr[0]), int(hdr[1]), int(hdr[4])
    return ({"segments": n_segs, "cut_items": n_comb, "pieces": int(hdr[2]), "heads": int(hdr[3]),
             "empty_items": n_empty},
            b[off_seg_begin:off_seg_begin + 4 * (G + 1)].view(np.int32),
            b[off_segs:off_segs + 16 * n_segs].view(np.int32).reshape(n_segs, 4),
            b[off_comb:off_comb + 16 * n_comb].view(np.int32).reshape(n_comb, 4),
            b[off_empties:off_empties + 4 * n_empty].view(np.int32))


def block_sparse_attention_scheduled(q, k, v, kidx, kcnt, geom: Geometry, item_begin: int, item_count: int, out,
                                     schedule, stream=None):
    """block_sparse_attention_range over a schedule from make_schedule (same kcnt and range): the persistent bf16
    kernel, then the merge of cut items and the zeros of empty ones (the fp32 lane runs the per-item kernel)."""
    q2, k2, v2, o2 = _rows(q), _rows(k), _rows(v), _rows(out)
    g = Geometry(**{**geom.__dict__, "dtype": _dtype_code(q2)})
    p = g.params()
    _check(lib().fvsr_lcsa_attention_scheduled(ctypes.byref(p), _ptr(q2), _ptr(k2), _ptr(v2), _ptr(kidx), _ptr(kcnt),
                                               _ptr(o2), int(item_begin), int(item_count), _ptr(schedule),
                                               schedule.numel(), _stream(stream)))
    return out


@dataclass
class Shard:
    """One rank's share of a (head, query block) item space split across GPUs: global items [begin, end), the heads
    they touch [head_lo, head_hi], and the range relative to those heads (what the rank's local tensors index)."""
    begin: int
    end: int
    head_lo: int
    head_hi: int

    @property
    def heads(self) -> int:
        return self.head_hi - self.head_lo + 1

    def local_range(self, nq: int) -> tuple[int, int]:
        return self.begin - self.head_lo * nq, self.end - self.begin


def shard_items(heads: int, nq: int, world: int, rank: int) -> Shard:
    """Contiguous, balanced split of the H·Nq head-major work items. A rank needs the Q/K/V of every head it touches
    (selection is joint over all query blocks of a (head, slice) row), so heads shared by two ranks are computed by
    both; attention runs only on the rank's own items."""
    total = heads * nq
    b = total * rank // world
    e = total * (rank + 1) // world
    if e <= b:
        return Shard(b, b, 0, -1)
    return Shard(b, e, b // nq, (e - 1) // nq)


def kernel_block_attention(q, k, v, block_mask, heads: int, workspace=None, stream=None):
    """kernelBlockAttention(q:k:v:blockMask:heads:) (SparseAttention.swift:169-187). q (1, Lq, H·128), k / v
    (1, Lk, H·128) window order, block_mask (H, Nq, Nk) 0/1 (kept where > 0.5). Returns (1, Lq, H·128)."""
    torch = _torch()
    shape = q.shape
    q2, k2, v2 = _rows(q), _rows(k), _rows(v)
    if q2.shape[1] != heads * 128:
        raise FVSRError(FVSR_EINVAL, "kernel attention: batch 1, head dim 128")
    nq, nk = block_mask.shape[1], block_mask.shape[2]
    g = Geometry(heads=heads, bh=1, bw=1, q_slices=nq, kv_slices=nk, local_range=1, topk=0, dtype=_dtype_code(q2))
    bm = block_mask.to(torch.float32).contiguous()
    out = torch.empty_like(q2)
    ws = workspace if workspace is not None else make_workspace(g, q2.device)
    p = g.params()
    _check(lib().fvsr_lcsa_attention_mask(ctypes.byref(p), _ptr(q2), _ptr(k2), _ptr(v2), _ptr(bm), _ptr(out),
                                          _ptr(ws), ws.numel(), _stream(stream)))
    return out.reshape(shape)


class FlashVSRAttentionOps:
    """The public kernel entry point of SparseAttention.swift:190-201. The reference offers the same meaning in three
    lanes; `kernel` is the one this path replaces (the sm_100a kernels). Its `dense` and `gathered` lanes are study
    code (Sources/Smoke/Diag.swift:86-121 compares them) and are not offered here."""

    @staticmethod
    def kernel(q, k, v, block_mask, heads: int, simdgroups: int | None = None):
        """`simdgroups` is the Metal kernel's threadgroup size (SparseAttention.swift:169-170); it has no B200
        counterpart (one tcgen05 CTA per work item) and is accepted for call compatibility only."""
        if simdgroups is not None and simdgroups < 1:
            raise FVSRError(FVSR_EINVAL, "simdgroups must be >= 1")
        return kernel_block_attention(q, k, v, block_mask, heads)


class KVCache:
    """The window K/V cache of blockForward (DiT.swift:507-511, 532-538) as slice pages appended in place."""

    def __init__(self, geom: Geometry, kv_len: int, max_new_slices: int, page_blocks: int | None = None):
        """page_blocks: arena blocks per page (default s); more leaves room for N equal gathered shards."""
        self.geom = geom
        self.kv_len = kv_len
        self.capacity = kv_len + max_new_slices
        self.page_blocks = page_blocks or geom.s
        h = ctypes.c_void_p()
        p = geom.params()
        _check(lib().fvsr_kv_cache_create_padded(ctypes.byref(p), kv_len, max_new_slices, self.page_blocks,
                                                 ctypes.byref(h)))
        self.handle = h

    def close(self):
        if self.handle:
            lib().fvsr_kv_cache_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reset(self):
        _check(lib().fvsr_kv_cache_reset(self.handle))

    @property
    def slices(self) -> int:
        n = ctypes.c_int32(0)
        _check(lib().fvsr_kv_cache_slices(self.handle, ctypes.byref(n)))
        return int(n.value)

    def append(self, k_new, v_new, new_slices: int, stream=None):
        _check(lib().fvsr_kv_cache_append(self.handle, _ptr(_rows(k_new)), _ptr(_rows(v_new)), new_slices,
                                          _stream(stream)))

    def trim(self):
        _check(lib().fvsr_kv_cache_trim(self.handle))

    def reserve(self):
        """The next free page as device views (k (page_blocks·128, H·128), v likewise, pooled k (page_blocks, H·128)
        fp32), for a collective to fill; commit() then appends it as the newest slice."""
        torch = _torch()
        k, v, pk = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
        _check(lib().fvsr_kv_cache_reserve(self.handle, ctypes.byref(k), ctypes.byref(v), ctypes.byref(pk)))
        rows, c = self.page_blocks * 128, self.geom.channels
        dt, code = (torch.bfloat16, "<i2") if self.geom.dtype == FVSR_BF16 else (torch.float32, "<f4")
        views = []
        for ptr, shape, tcode, tdt in ((k, (rows, c), code, dt), (v, (rows, c), code, dt),
                                       (pk, (self.page_blocks, c), "<f4", torch.float32)):
            t = torch.as_tensor(_DeviceArray(ptr.value, shape, tcode), device="cuda")
            views.append(t.view(tdt) if tdt == torch.bfloat16 else t)
        return tuple(views)

    def commit(self):
        _check(lib().fvsr_kv_cache_commit(self.handle))

    def state(self) -> list[int]:
        n = ctypes.c_int32(0)
        buf = (ctypes.c_int32 * self.capacity)()
        _check(lib().fvsr_kv_cache_state(self.handle, buf, ctypes.byref(n)))
        return list(buf[: n.value])

    def gather(self, stream=None):
        torch = _torch()
        n = self.slices
        rows = n * self.geom.s * 128
        dt = torch.bfloat16 if self.geom.dtype == FVSR_BF16 else torch.float32
        k = torch.empty((rows, self.geom.channels), dtype=dt, device="cuda")
        v = torch.empty_like(k)
        _check(lib().fvsr_kv_cache_gather(self.handle, _ptr(k), _ptr(v), _stream(stream)))
        return k, v


def lcsa_forward(q, k_new, v_new, cache: KVCache, geom: Geometry, out=None, kidx=None, kcnt=None, workspace=None,
                 stream=None):
    """One streaming layer (DiT.swift:504-538): append (k_new, v_new), select over cache ⊕ current, attend, trim.
    geom.q_slices = the chunk's slices; geom.kv_slices is ignored (taken from the cache)."""
    torch = _torch()
    q2 = _rows(q)
    if out is None:
        out = torch.empty_like(q2)
    full = Geometry(**{**geom.__dict__, "kv_slices": min(cache.slices + geom.q_slices, cache.capacity)})
    ws = workspace if workspace is not None else make_workspace(full, q2.device)
    p = geom.params()
    _check(lib().fvsr_lcsa_forward(ctypes.byref(p), _ptr(q2), _ptr(_rows(k_new)), _ptr(_rows(v_new)), cache.handle,
                                   _ptr(out), _ptr(kidx), _ptr(kcnt), _ptr(ws), ws.numel(), _stream(stream)))
    return out


@dataclass(frozen=True)
class QueryShard:
    """One rank's query blocks of a chunk split across `world` GPUs: [begin, end) of the chunk's nq windows, and the
    equal padded shard of `width` blocks every rank contributes to a gather (world·width ≥ nq; the last ranks' shards
    may hold fewer real blocks, and a rank past the end holds none)."""
    begin: int
    end: int
    width: int

    @property
    def blocks(self) -> int:
        return self.end - self.begin


def query_shard(nq: int, world: int, rank: int) -> QueryShard:
    """Contiguous split of a chunk's nq query blocks into shards of width = ceil(nq / world) blocks, in rank order —
    the layout a sequence-split QKV projection leaves, and the one an all-gather of equal shards reassembles."""
    if world < 1 or not 0 <= rank < world or nq < 1:
        raise FVSRError(FVSR_EINVAL, f"bad shard request nq={nq} world={world} rank={rank}")
    width = -(-nq // world)
    b = min(nq, rank * width)
    return QueryShard(b, min(nq, b + width), width)


def lcsa_forward_shard(q, shard: QueryShard, pooled_q, cache: KVCache, geom: Geometry, out=None, kv_ready=None,
                       kidx=None, kcnt=None, workspace=None, stream=None):
    """One rank's layer call (fvsr_lcsa_forward_shard): the full selection over pooled_q (Nq, H·128) fp32 and the
    cache's pooled keys (the current slice committed), then the attention of the rank's query blocks over every head
    after `kv_ready` (a torch.cuda.Event recorded when the K/V gather into the page is done), then the trim.
    q / out: (shard.blocks·128, H·128) window order."""
    torch = _torch()
    q2 = _rows(q)
    if out is None:
        out = torch.empty_like(q2)
    full = Geometry(**{**geom.__dict__, "kv_slices": cache.slices})
    ws = workspace if workspace is not None else make_workspace(full, q2.device)
    p = geom.params()
    ev = None if kv_ready is None else ctypes.c_void_p(kv_ready.cuda_event)
    _check(lib().fvsr_lcsa_forward_shard(ctypes.byref(p), _ptr(q2), shard.begin, shard.end, _ptr(pooled_q),
                                         cache.handle, ev, _ptr(_rows(out)), _ptr(kidx), _ptr(kcnt), _ptr(ws),
                                         ws.numel(), _stream(stream)))
    return out


def partial_size(geom: Geometry, shard: QueryShard) -> int:
    """Bytes of the fp32 partial results lcsa_attend_shard keeps between its two launches."""
    n = ctypes.c_size_t(0)
    p = geom.params()
    _check(lib().fvsr_lcsa_partial_size(ctypes.byref(p), shard.begin, shard.end, ctypes.byref(n)))
    return int(n.value)


def lcsa_select_shard(pooled_q, shard: QueryShard, cache: KVCache, geom: Geometry, workspace, kidx=None, kcnt=None,
                      spare_sms: int = 0, stream=None):
    """The selection of a rank's layer call (fvsr_lcsa_select_shard): over pooled_q and the cache's pooled keys (the
    current slice committed), with the longest-first order of the rank's items kept in the workspace. spare_sms:
    SMs left free for a collective running beside it."""
    p = geom.params()
    _check(lib().fvsr_lcsa_select_shard(ctypes.byref(p), _ptr(pooled_q), shard.begin, shard.end, cache.handle,
                                        _ptr(kidx), _ptr(kcnt), _ptr(workspace), workspace.numel(), int(spare_sms),
                                        _stream(stream)))


def lcsa_attend_shard(q, shard: QueryShard, cache: KVCache, geom: Geometry, workspace, out, kv_ready=None,
                      partial=None, kidx=None, kcnt=None, stream=None):
    """The attention of a rank's layer call (fvsr_lcsa_attend_shard): with `partial`, the cached slices' blocks
    first, then — after kv_ready — the current slice's, merged; then the trim."""
    p = geom.params()
    ev = None if kv_ready is None else ctypes.c_void_p(kv_ready.cuda_event)
    _check(lib().fvsr_lcsa_attend_shard(ctypes.byref(p), _ptr(_rows(q)), shard.begin, shard.end, cache.handle, ev,
                                        _ptr(partial), 0 if partial is None else partial.numel(), _ptr(_rows(out)),
                                        _ptr(kidx), _ptr(kcnt), _ptr(workspace), workspace.numel(), _stream(stream)))
    return out


def _bf16_2d(t, name):
    torch = _torch()
    if t.dtype != torch.bfloat16 or t.dim() != 2 or not t.is_cuda or not t.is_contiguous():
        raise FVSRError(FVSR_EINVAL, f"{name} must be a contiguous 2-D bf16 CUDA tensor")
    return t


def linear(x, w, bias=None, epilogue: int = FVSR_LINEAR, gate=None, resid=None, out=None, stream=None):
    """MLX's Linear on the tensor cores (fvsr_linear): x (M, K) · w (N, K)ᵀ + bias, bf16, with the epilogue
    FVSR_LINEAR, FVSR_LINEAR_GELU (GELU(tanh) of it) or FVSR_LINEAR_GATED_RESIDUAL (resid + gate · it)."""
    torch = _torch()
    x, w = _bf16_2d(_rows(x), "x"), _bf16_2d(w, "w")
    m, k = x.shape
    n = w.shape[0]
    if w.shape[1] != k:
        raise FVSRError(FVSR_EINVAL, f"w must be ({n}, {k})")
    if out is None:
        out = torch.empty((m, n), dtype=torch.bfloat16, device=x.device)
    _check(lib().fvsr_linear(m, n, k, _ptr(x), _ptr(w), _ptr(bias), int(epilogue), _ptr(gate), _ptr(resid),
                             _ptr(out), _stream(stream)))
    return out


def linear_qkv(x, w, bias=None, outs=None, stream=None):
    """The q, k, v projections in one launch (fvsr_linear_qkv): w = [Wq; Wk; Wv] (3n, K) → three (M, n) tensors."""
    torch = _torch()
    x, w = _bf16_2d(_rows(x), "x"), _bf16_2d(w, "w")
    m, k = x.shape
    n = w.shape[0] // 3
    if outs is None:
        outs = tuple(torch.empty((m, n), dtype=torch.bfloat16, device=x.device) for _ in range(3))
    _check(lib().fvsr_linear_qkv(m, n, k, _ptr(x), _ptr(w), _ptr(bias), _ptr(outs[0]), _ptr(outs[1]),
                                 _ptr(outs[2]), _stream(stream)))
    return outs


def layernorm(x, weight=None, bias=None, shift=None, scale=None, eps: float = 1e-6, out=None, stream=None):
    """LayerNorm over the channels (fvsr_layernorm): norm1/norm2 (no affine) with the block's modulation
    y·(1 + scale) + shift when shift and scale are given (DiT.swift:489-494, 546); norm3 with weight and bias."""
    torch = _torch()
    x = _bf16_2d(_rows(x), "x")
    if out is None:
        out = torch.empty_like(x)
    _check(lib().fvsr_layernorm(x.shape[0], x.shape[1], _ptr(x), _ptr(weight), _ptr(bias), _ptr(shift), _ptr(scale),
                                float(eps), _ptr(out), _stream(stream)))
    return out


def rmsnorm(x, weight, eps: float = 1e-6, out=None, stream=None):
    """WanRMSNorm (DiT.swift:34-47) of each row (fvsr_rmsnorm)."""
    torch = _torch()
    x = _bf16_2d(_rows(x), "x")
    if out is None:
        out = torch.empty_like(x)
    _check(lib().fvsr_rmsnorm(x.shape[0], x.shape[1], _ptr(x), _ptr(weight), float(eps), _ptr(out), _stream(stream)))
    return out


def cross_attention(q, k, v, heads: int, out=None, stream=None):
    """The cross-attention core (DiT.swift:351-360, fvsr_cross_attention): every query over all context keys."""
    torch = _torch()
    q, k, v = (_bf16_2d(_rows(t), n) for t, n in ((q, "q"), (k, "k"), (v, "v")))
    if out is None:
        out = torch.empty_like(q)
    _check(lib().fvsr_cross_attention(int(heads), q.shape[0], k.shape[0], _ptr(q), _ptr(k), _ptr(v), _ptr(out),
                                      _stream(stream)))
    return out


def rope_tables(f: int, h: int, w: int, t0: int = 0, head_dim: int = 128, theta: float = 10000.0, device="cuda"):
    """RopeTables (DiT.swift:52-97): for every token of an (f, h, w) patch grid in token order, temporal positions
    starting at t0, the 64 (cos, sin) entries of the 3-D factorised rotation — temporal 44 | height 42 | width 42 of a
    128-wide head, each axis's frequencies normalised by its own sub-dimension, angles in float64, tables in fp32.
    Returns (cos, sin), each (f·h·w, 64) fp32."""
    import numpy as np
    torch = _torch()
    if head_dim != 128:
        raise FVSRError(FVSR_EINVAL, "head_dim must be 128")
    if t0 < 0 or t0 + f > 1024 or h > 1024 or w > 1024:
        raise FVSRError(FVSR_EINVAL, "positions must stay below 1024 (RopeTables.end)")
    d_hw = head_dim // 3
    d_t = head_dim - 2 * d_hw

    def table(dim, positions):
        j = np.arange(dim // 2, dtype=np.float64)
        freq = 1.0 / np.power(theta, 2.0 * j / dim)
        ang = np.asarray(positions, dtype=np.float64)[:, None] * freq[None, :]
        return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)

    ct, st = table(d_t, np.arange(t0, t0 + f))
    ch, sh = table(d_hw, np.arange(h))
    cw, sw = table(d_hw, np.arange(w))

    def grid(tt, th, tw):
        n = tt.shape[1] + th.shape[1] + tw.shape[1]
        g = np.empty((f, h, w, n), np.float32)
        g[..., : tt.shape[1]] = tt[:, None, None, :]
        g[..., tt.shape[1]: tt.shape[1] + th.shape[1]] = th[None, :, None, :]
        g[..., tt.shape[1] + th.shape[1]:] = tw[None, None, :, :]
        return torch.from_numpy(g.reshape(f * h * w, n)).to(device)

    return grid(ct, ch, cw), grid(st, sh, sw)


def _token_inputs(geom: Geometry, q_lin, k_lin, v_lin, norm_q, norm_k, rope):
    rows = geom.nq * 128
    ts = [_rows(t) for t in (q_lin, k_lin, v_lin)]
    for t in ts:
        if t.shape != (rows, geom.channels):
            raise FVSRError(FVSR_EINVAL, f"linear outputs must be ({rows}, {geom.channels}), got {tuple(t.shape)}")
        if _dtype_code(t) != geom.dtype:
            raise FVSRError(FVSR_EINVAL, "q, k and v must all be in the geometry's dtype")
    for wt in (norm_q, norm_k):
        if wt is not None and (wt.dtype != ts[0].dtype or tuple(wt.shape) != (geom.channels,) or not wt.is_contiguous()
                               or not wt.is_cuda):
            raise FVSRError(FVSR_EINVAL, f"norm weights must be contiguous CUDA ({geom.channels},) in the q dtype")
    cos, sin = rope if rope is not None else (None, None)
    for t in (cos, sin):
        if t is not None and (t.dtype != _torch().float32 or tuple(t.shape) != (rows, 64) or not t.is_contiguous()):
            raise FVSRError(FVSR_EINVAL, f"rotation tables must be contiguous ({rows}, 64) fp32")
    return ts, cos, sin


def lcsa_prepare(q_lin, k_lin, v_lin, geom: Geometry, norm_q=None, norm_k=None, eps: float = 1e-6, rope=None,
                 pooled: bool = True, stream=None) -> dict:
    """The q/k/v side of one layer (DiT.swift:497-506) from the linear outputs (token order, (Nq·128, H·128)):
    WanRMSNorm of q and k (weights norm_q / norm_k, None = skipped), ropeApply with rope = (cos, sin) tables from
    rope_tables (None = skipped), windowPartition of all three, and the pooled q / k the selection reads.
    Returns {"q", "k", "v"} window-ordered and, with pooled, {"pooled_q", "pooled_k"} (Nq, H·128) fp32."""
    torch = _torch()
    (q, k, v), cos, sin = _token_inputs(geom, q_lin, k_lin, v_lin, norm_q, norm_k, rope)
    res = {"q": torch.empty_like(q), "k": torch.empty_like(k), "v": torch.empty_like(v)}
    if pooled:
        res["pooled_q"] = torch.empty((geom.nq, geom.channels), dtype=torch.float32, device=q.device)
        res["pooled_k"] = torch.empty_like(res["pooled_q"])
    p = geom.params()
    _check(lib().fvsr_lcsa_prepare(ctypes.byref(p), _ptr(q), _ptr(k), _ptr(v), _ptr(norm_q), _ptr(norm_k), eps,
                                   _ptr(cos), _ptr(sin), _ptr(res["q"]), _ptr(res["k"]), _ptr(res["v"]),
                                   _ptr(res.get("pooled_q")), _ptr(res.get("pooled_k")), _stream(stream)))
    return res


def lcsa_forward_tokens(q_lin, k_lin, v_lin, cache: KVCache, geom: Geometry, norm_q=None, norm_k=None,
                        eps: float = 1e-6, rope=None, q_win=None, out=None, kidx=None, kcnt=None, workspace=None,
                        stream=None):
    """One streaming layer from the linear outputs to the input of the output projection (DiT.swift:499-539):
    prepare (k, v straight into the cache), select over cache ⊕ current, attend, trim; returns the output in token
    order (windowReverse fused). geom.q_slices = the chunk's slices; geom.kv_slices is taken from the cache."""
    torch = _torch()
    (q, k, v), cos, sin = _token_inputs(geom, q_lin, k_lin, v_lin, norm_q, norm_k, rope)
    if q_win is None:
        q_win = torch.empty_like(q)
    if out is None:
        out = torch.empty_like(q)
    full = Geometry(**{**geom.__dict__, "kv_slices": min(cache.slices + geom.q_slices, cache.capacity)})
    ws = workspace if workspace is not None else make_workspace(full, q.device)
    p = geom.params()
    _check(lib().fvsr_lcsa_forward_tokens(ctypes.byref(p), _ptr(q), _ptr(k), _ptr(v), _ptr(norm_q), _ptr(norm_k), eps,
                                          _ptr(cos), _ptr(sin), cache.handle, _ptr(q_win), _ptr(out), _ptr(kidx),
                                          _ptr(kcnt), _ptr(ws), ws.numel(), _stream(stream)))
    return out


def chunk_geometry(k: int, heads: int, out_h: int, out_w: int, dtype: int = FVSR_BF16, topk_ratio: float = 0.0,
                   local_range: int = 11):
    """The step geometry of streaming chunk k (Pipeline.swift:95-102, DiT.swift:478-485), host only:
    (Geometry, latent_begin, latent_end); latent_begin is the chunk's RoPE temporal start t0."""
    p = Params()
    b, e = ctypes.c_int32(0), ctypes.c_int32(0)
    _check(lib().fvsr_stream_chunk_geometry(heads, out_h, out_w, dtype, float(topk_ratio), local_range, k,
                                            ctypes.byref(p), ctypes.byref(b), ctypes.byref(e)))
    g = Geometry(heads=p.heads, bh=p.bh, bw=p.bw, q_slices=p.q_slices, kv_slices=p.kv_slices,
                 local_range=p.local_range, topk=p.topk, dtype=p.dtype)
    return g, int(b.value), int(e.value)


class _DeviceArray:
    """A device buffer of the library seen by torch through __cuda_array_interface__ (fp32 "<f4" or 16-bit "<i2")."""

    def __init__(self, ptr: int, shape: tuple, typestr: str = "<f4"):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False), "version": 2,
                                         "strides": None}


class Stream:
    """The LCSA side of FlashVSR's chunk loop (FlashVSRPipeline.chunk / FlashVSRDiT.step, Pipeline.swift:95-131,
    DiT.swift:554-578) for `layers` DiT blocks at an output size out_h × out_w: chunk schedule, RoPE tables per chunk,
    topk, kvLen = int(kv_ratio), one window cache per block. Call begin(), then for k = 0, 1, …: start_chunk(k) and
    layer(i, q, k, v, norm_q, norm_k) for each block i."""

    def __init__(self, heads: int, out_h: int, out_w: int, layers: int, dtype: int = FVSR_BF16,
                 topk_ratio: float = 0.0, kv_ratio: float = 3.0, local_range: int = 11):
        h = ctypes.c_void_p()
        _check(lib().fvsr_stream_create(heads, out_h, out_w, layers, dtype, float(topk_ratio), float(kv_ratio),
                                        local_range, ctypes.byref(h)))
        self.handle = h
        self.heads, self.out_h, self.out_w, self.layers, self.dtype = heads, out_h, out_w, layers, dtype
        self.topk_ratio, self.local_range = topk_ratio, local_range
        self.chunk = -1
        n = ctypes.c_size_t(0)
        _check(lib().fvsr_stream_workspace_size(self.handle, ctypes.byref(n)))
        self.workspace = _torch().empty(int(n.value), dtype=_torch().uint8, device="cuda")

    def close(self):
        if self.handle:
            lib().fvsr_stream_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def begin(self):
        _check(lib().fvsr_stream_begin(self.handle))
        self.chunk = -1

    def geometry(self, k: int):
        return chunk_geometry(k, self.heads, self.out_h, self.out_w, self.dtype, self.topk_ratio, self.local_range)

    def start_chunk(self, k: int, stream=None):
        _check(lib().fvsr_stream_start_chunk(self.handle, k, _stream(stream)))
        self.chunk = k

    def rope(self):
        """The current chunk's (tokens, 64) fp32 RoPE tables, copied out of the stream."""
        torch = _torch()
        c, s, n = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_int64(0)
        _check(lib().fvsr_stream_rope(self.handle, ctypes.byref(c), ctypes.byref(s), ctypes.byref(n)))
        out = []
        for ptr in (c, s):
            view = _DeviceArray(ptr.value, (int(n.value), 64))
            out.append(torch.as_tensor(view, device="cuda").clone())
        return tuple(out)

    def layer(self, i: int, q_lin, k_lin, v_lin, norm_q=None, norm_k=None, eps: float = 1e-6, q_win=None, out=None,
              kidx=None, kcnt=None, stream=None):
        torch = _torch()
        g, _, _ = self.geometry(self.chunk)
        (q, k, v), _, _ = _token_inputs(g, q_lin, k_lin, v_lin, norm_q, norm_k, None)
        q_win = torch.empty_like(q) if q_win is None else q_win
        out = torch.empty_like(q) if out is None else out
        _check(lib().fvsr_stream_layer(self.handle, i, _ptr(q), _ptr(k), _ptr(v), _ptr(norm_q), _ptr(norm_k), eps,
                                       _ptr(q_win), _ptr(out), _ptr(kidx), _ptr(kcnt), _ptr(self.workspace),
                                       self.workspace.numel(), _stream(stream)))
        return out


def wait_probe(limit_us: int, stream=None) -> None:
    """Runs one bounded device wait that nothing completes (fvsr_wait_probe); the next device_check raises
    FVSRError(FVSR_ETIMEOUT). The failure path of the attention kernels' waits, exercised without a fault."""
    _check(lib().fvsr_wait_probe(int(limit_us), _stream(stream)))


def device_check(stream=None) -> None:
    """Synchronise and raise FVSRError(FVSR_ETIMEOUT) if a device-side wait of this library gave up."""
    _check(lib().fvsr_device_check(_stream(stream)))
