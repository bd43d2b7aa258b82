"""Python face of the CPU oracle (``oracle/fvsr_oracle.c``) — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg import this module, and only as the
checker or as the timed CPU baseline; the product library never loads it.

All arrays are numpy, C-contiguous. bf16 tensors travel as ``uint16`` bit patterns.
Reference citations are relative to the xocialize/mlx-flashvsr-swift tree.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "libfvsr_oracle.so"
BLOCK = 128
D = 128

_lib = None


def build() -> Path:
    """Compile the oracle with its Makefile (gcc + OpenMP)."""
    subprocess.run(["make", "-C", str(HERE)], check=True, stdout=subprocess.DEVNULL)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        _lib = ctypes.CDLL(str(LIB_PATH))
        P, I, I64, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
        _lib.fvsr_exp.argtypes = [F]
        _lib.fvsr_exp.restype = F
        _lib.orc_window_partition.argtypes = [P, I, I, I, I, I, P]
        _lib.orc_window_reverse.argtypes = [P, I, I, I, I, I, P]
        _lib.orc_prepare.argtypes = [P, I, I, I, I, I, P, F, P, P, P]
        _lib.orc_local_block_mask.argtypes = [I, I, I, P]
        _lib.orc_local_block_mask.restype = None
        _lib.orc_geometry_topk.argtypes = [I, ctypes.c_double]
        _lib.orc_pool.argtypes = [P, I, I64, I64, P]
        _lib.orc_pool.restype = None
        _lib.orc_select.argtypes = [I, I, I, I, I, P, I, P, P, P, P, P, P]
        _lib.orc_mask_to_lists.argtypes = [P, I, I, I, P, P]
        _lib.orc_mask_to_lists.restype = None
        for name in ("orc_attention", "orc_attention_fast"):
            fn = getattr(_lib, name)
            fn.argtypes = [I, P, P, P, I, I, I, P, P, P, I64, P]
            fn.restype = None
        _lib.orc_num_threads.restype = I
        _lib.orc_set_num_threads.argtypes = [I]
        _lib.orc_set_num_threads.restype = None
    return _lib


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _dtype_code(x: np.ndarray) -> int:
    if x.dtype == np.float32:
        return 0
    if x.dtype == np.uint16:
        return 1
    raise TypeError(f"oracle takes float32 or bf16-as-uint16, got {x.dtype}")


# ---------------------------------------------------------------------------------------------------------------
# bf16 helpers (round to nearest even, the conversion torch and MLX use)
# ---------------------------------------------------------------------------------------------------------------

def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return rounded.astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---------------------------------------------------------------------------------------------------------------
# Restated reference functions
# ---------------------------------------------------------------------------------------------------------------

def fvsr_exp(x: float) -> float:
    return lib().fvsr_exp(float(x))


def window_partition(x: np.ndarray) -> np.ndarray:
    """DiT.swift:113-118. x (B, F, H, W, C) fp32 → (B·F/2·H/8·W/8, 128, C)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    b, f, h, w, c = x.shape
    out = np.empty(((b * (f // 2) * (h // 8) * (w // 8)), 128, c), np.float32)
    if lib().orc_window_partition(_p(x), b, f, h, w, c, _p(out)) != 0:
        raise ValueError("window partition needs F even and H, W multiples of 8")
    return out


def window_reverse(x: np.ndarray, b: int, f: int, h: int, w: int) -> np.ndarray:
    """DiT.swift:121-126. Inverse of window_partition → (B, F·H·W, C)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    c = x.shape[-1]
    out = np.empty((b, f * h * w, c), np.float32)
    if lib().orc_window_reverse(_p(x), b, f, h, w, c, _p(out)) != 0:
        raise ValueError("window reverse needs F even and H, W multiples of 8")
    return out


def prepare(x: np.ndarray, f: int, h: int, w: int, heads: int, weight: np.ndarray | None = None, eps: float = 1e-6,
            cos: np.ndarray | None = None, sin: np.ndarray | None = None) -> np.ndarray:
    """DiT.swift:34-47, 100-107, 113-118: x (F·H·W, heads·128) token order, fp32 or bf16 bits → WanRMSNorm (weight
    given) → ropeApply (cos/sin (F·H·W, 64) fp32 given) → window order, same dtype, with the storage-type rounding
    points of the reference (see orc_prepare)."""
    x = np.ascontiguousarray(x)
    dt = _dtype_code(x)
    if weight is not None:
        weight = np.ascontiguousarray(weight, dtype=x.dtype)
    if (cos is None) != (sin is None):
        raise ValueError("cos and sin go together")
    if cos is not None:
        cos = np.ascontiguousarray(cos, dtype=np.float32)
        sin = np.ascontiguousarray(sin, dtype=np.float32)
    out = np.empty_like(x)
    if lib().orc_prepare(_p(x), dt, f, h, w, heads, _p(weight), float(eps), _p(cos), _p(sin), _p(out)) != 0:
        raise ValueError("prepare needs F even and H, W multiples of 8")
    return out


def local_block_mask(bh: int, bw: int, r: int) -> np.ndarray:
    """DiT.swift:130-145 → (s, s) bool, s = bh·bw."""
    s = bh * bw
    out = np.empty((s, s), np.uint8)
    lib().orc_local_block_mask(bh, bw, r, _p(out))
    return out.astype(bool)


def geometry_topk(s: int, ratio: float) -> int:
    """DiT.swift:482: topk = Int(Double(s·s)·ratio) − 1."""
    return int(lib().orc_geometry_topk(s, ratio))


def pool(x: np.ndarray) -> np.ndarray:
    """DiT.swift:161-162. x (N·128, C) fp32 or bf16 bits → (N, C) fp32 block means in the fixed order."""
    x = np.ascontiguousarray(x)
    rows, c = x.shape
    assert rows % BLOCK == 0
    out = np.empty((rows // BLOCK, c), np.float32)
    lib().orc_pool(_p(x), _dtype_code(x), rows // BLOCK, c, _p(out))
    return out


def select(pq: np.ndarray, pk: np.ndarray, heads: int, q_slices: int, s: int, local: np.ndarray, topk: int):
    """DiT.swift:158-174 on pooled inputs. pq (Nq, H·128), pk (Nk, H·128) fp32; local (s, s) bool.
    Returns (probs (H,Nq,Nk) f32, mask (H,Nq,Nk) bool, kidx (H,Nq,Nk) i32, kcnt (H,Nq) i32)."""
    pq = np.ascontiguousarray(pq, dtype=np.float32)
    pk = np.ascontiguousarray(pk, dtype=np.float32)
    nq, nk = pq.shape[0], pk.shape[0]
    loc = np.ascontiguousarray(local, dtype=np.uint8)
    probs = np.empty((heads, nq, nk), np.float32)
    mask = np.empty((heads, nq, nk), np.uint8)
    kidx = np.empty((heads, nq, nk), np.int32)
    kcnt = np.empty((heads, nq), np.int32)
    rc = lib().orc_select(heads, nq, nk, s, q_slices, _p(loc), topk, _p(pq), _p(pk), _p(probs), _p(mask),
                          _p(kidx), _p(kcnt))
    if rc != 0:
        raise ValueError("bad selection shape")
    return probs, mask.astype(bool), kidx, kcnt


def draft_block_mask_and_probs(q: np.ndarray, k: np.ndarray, heads: int, q_slices: int, s: int, local: np.ndarray,
                               topk: int):
    """DiT.swift:158-174 end to end: q (Lq, H·128), k (Lk, H·128) fp32 or bf16 bits in window order."""
    return select(pool(q), pool(k), heads, q_slices, s, local, topk)


def mask_to_lists(mask: np.ndarray):
    """SparseAttention.swift:175-177 with ascending order. mask (H, Nq, Nk) 0/1 → (kidx, kcnt)."""
    m = np.ascontiguousarray(mask, dtype=np.float32)
    h, nq, nk = m.shape
    kidx = np.empty((h, nq, nk), np.int32)
    kcnt = np.empty((h, nq), np.int32)
    lib().orc_mask_to_lists(_p(m), h, nq, nk, _p(kidx), _p(kcnt))
    return kidx, kcnt


def attention(q, k, v, kidx, kcnt, heads: int, items=None, fast: bool = False) -> np.ndarray:
    """Softmax attention over the kept blocks (DiT.swift:279-313). q (Lq, H·128), k/v (Lk, H·128) fp32 or bf16
    bits; kidx/kcnt from select/mask_to_lists; items = optional list of h·Nq + qb to evaluate (others left 0)."""
    q, k, v = (np.ascontiguousarray(a) for a in (q, k, v))
    dt = _dtype_code(q)
    assert _dtype_code(k) == dt and _dtype_code(v) == dt
    kidx = np.ascontiguousarray(kidx, dtype=np.int32)
    kcnt = np.ascontiguousarray(kcnt, dtype=np.int32)
    nq, nk = kidx.shape[1], kidx.shape[2]
    out = np.zeros((q.shape[0], q.shape[1]), np.float32)
    it = None if items is None else np.ascontiguousarray(items, dtype=np.int32)
    n_items = 0 if it is None else len(it)
    fn = lib().orc_attention_fast if fast else lib().orc_attention
    fn(dt, _p(q), _p(k), _p(v), heads, nq, nk, _p(kidx), _p(kcnt), _p(it), n_items, _p(out))
    return out


def set_num_threads(n: int) -> None:
    lib().orc_set_num_threads(int(n))


def num_threads() -> int:
    return int(lib().orc_num_threads())


# ---------------------------------------------------------------------------------------------------------------
# Comparison helpers following the reference's gate receipts
# ---------------------------------------------------------------------------------------------------------------

def compare(got: np.ndarray, ref: np.ndarray) -> dict:
    """Sources/Smoke/Gates.swift:19-29: maxAbs, ref |max|, rel = maxAbs / ref|max|, PSNR."""
    g = np.asarray(got, np.float64)
    r = np.asarray(ref, np.float64)
    d = np.abs(g - r)
    max_abs = float(d.max()) if d.size else 0.0
    ref_max = float(np.abs(r).max()) if r.size else 0.0
    peak = max(ref_max, 1e-12)
    mse = float((d * d).mean()) if d.size else 0.0
    psnr = float("inf") if mse == 0 else 10 * np.log10(peak * peak / mse)
    return {"max_abs": max_abs, "ref_max": ref_max, "rel": max_abs / peak, "psnr": psnr}


def pool_f64(x: np.ndarray, chunk_blocks: int = 256) -> np.ndarray:
    """DiT.swift:161-162 in float64: x (N·128, C) fp32 or bf16 bits → (N, C) float64 block means, a chunk of blocks
    at a time (a float64 copy of a whole config-5 key tensor would take over 1 GB)."""
    x = np.ascontiguousarray(x)
    if x.dtype == np.uint16:
        x = bf16_bits_to_f32(x).reshape(x.shape)
    n, c = x.shape[0] // BLOCK, x.shape[1]
    out = np.empty((n, c), np.float64)
    for b0 in range(0, n, chunk_blocks):
        b1 = min(n, b0 + chunk_blocks)
        out[b0:b1] = x[b0 * BLOCK:b1 * BLOCK].reshape(b1 - b0, BLOCK, c).astype(np.float64).mean(axis=1)
    return out


def select_f64(q: np.ndarray, k: np.ndarray, heads: int, q_slices: int, s: int, local: np.ndarray, topk: int,
               pooled: tuple | None = None):
    """draftBlockMaskAndProbs (DiT.swift:158-174) evaluated in float64, one step per reference line, with the exact
    (k+1)-th largest of each (head, slice) row from a full partition — an order-independent reference for the fp32
    mask. q (Lq, C), k (Lk, C) window order (or pooled = (pq, pk) float64 block means). Returns (mask (H,Nq,Nk) bool,
    probs (H,Nq,Nk) float64)."""
    pq, pk = pooled if pooled is not None else (pool_f64(q), pool_f64(k))                            # 161-162
    nq, nk = pq.shape[0], pk.shape[0]
    d = pq.shape[1] // heads
    pqh = pq.reshape(nq, heads, d).transpose(1, 0, 2)
    pkh = pk.reshape(nk, heads, d).transpose(1, 0, 2)
    scores = np.matmul(pqh, pkh.transpose(0, 2, 1)) / np.sqrt(d)                                      # 163
    lm = np.where(np.asarray(local, bool), 0.0, -np.inf)                                              # 165
    scores = scores + np.broadcast_to(lm.reshape(1, s, 1, s), (nq // s, s, nk // s, s)).reshape(nq, nk)  # 166-167
    e = np.exp(scores - scores.max(axis=-1, keepdims=True))
    probs = e / e.sum(axis=-1, keepdims=True)                                                         # 168
    flat = probs.reshape(heads * q_slices, (nq // q_slices) * nk)                                     # 169
    n = flat.shape[1]
    kk = min(n - 1, topk)                                                                             # 171
    thr = np.partition(flat, n - 1 - kk, axis=1)[:, n - 1 - kk:n - kk]                               # 172
    return (flat > thr).reshape(heads, nq, nk), probs                                                 # 173


def mask_flip_report(mine: np.ndarray, other: np.ndarray, probs: np.ndarray, q_slices: int) -> dict:
    """Sources/Smoke/Gates.swift:242-277: count mask flips and classify each as a near-tie — probability within 1e-3
    (relative) of its nearest sorted neighbour in the (head, slice) row, or below 1e-30."""
    h, nq, nk = probs.shape
    flat = probs.reshape(h * q_slices, (nq // q_slices) * nk)
    flips = (mine != other).reshape(flat.shape)
    n_flip = int(flips.sum())
    worst_gap, underflow = 0.0, 0
    for r in np.nonzero(flips.any(axis=1))[0]:
        row = flat[r]
        srt = np.sort(row)
        for c in np.nonzero(flips[r])[0]:
            p = row[c]
            if p < 1e-30:
                underflow += 1
                continue
            idx = int(np.searchsorted(srt, p))
            lo = srt[idx - 1] if idx > 0 else p
            hi = srt[idx + 1] if idx + 1 < len(srt) else p
            worst_gap = max(worst_gap, min(abs(p - lo), abs(hi - p)) / max(p, 1e-38))
    return {"flips": n_flip, "underflow": underflow, "worst_gap": worst_gap}
