"""Generate the committed golden fixtures under tests/golden/ (run once, in a container that holds the reference).

Attention fixtures (``attn_*.npz``): outputs of the REFERENCE'S OWN attention oracle,
``oracle/block_sparse_attn.py:block_sparse_attn_func`` of xocialize/mlx-flashvsr-swift (torch, CPU, fp32: dense SDPA
under the token-expanded block mask, empty query blocks → 0), imported from the reference tree and run unmodified.
The inputs follow the reference's attention probe (Sources/Smoke/Diag.swift:86-98): random q/k/v, a random block mask
of a given density, one query block forced empty. Inputs are NOT stored: they are regenerated from the seeds by
``detrand.normal`` / ``detrand.uniform`` (numpy-version independent), so a fixture holds only the mask and the output.

Selection fixtures (``select_*.npz``): no runnable implementation of the reference's selection exists here (it is
Swift/MLX, Sources/FlashVSRMLX/DiT.swift:158-174), so these hold a float64 numpy evaluation that follows those lines
operation by operation (mean, matmul / sqrt(d), local mask, softmax, sort, strict threshold). They cross-check the
oracle's fixed-order fp32 restatement on inputs whose pooled scores are well separated (config-2 style block offsets).

Usage:  python tests/golden/make_golden.py --reference PATH_TO_REFERENCE_TREE
"""
from __future__ import annotations

import argparse
import importlib.util
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import detrand  # noqa: E402

ATTN_CASES = [
    # name, heads, nq, nk, density, seed, forced-empty (head, query block)
    ("attn_probe_a", 2, 3, 5, 0.5, 11, (0, 1)),
    ("attn_probe_b", 2, 2, 6, 0.3, 12, (1, 0)),
]

SELECT_CASES = [
    # name, heads, bh, bw, q_slices, kv_slices, local_range, keep fraction, seed
    ("select_c2_small", 2, 2, 3, 1, 3, 3, 0.6, 21),
    ("select_slices2", 2, 2, 2, 2, 4, 3, 0.3, 22),
]


def attn_inputs(heads, nq, nk, density, seed, empty):
    c = heads * 128
    q = detrand.normal(seed * 10 + 0, (nq * 128, c))
    k = detrand.normal(seed * 10 + 1, (nk * 128, c))
    v = detrand.normal(seed * 10 + 2, (nk * 128, c))
    mask = (detrand.uniform(seed * 10 + 3, (heads, nq, nk)) < density).astype(np.float32)
    mask[empty[0], empty[1], :] = 0
    return q, k, v, mask


def select_inputs(heads, bh, bw, q_slices, kv_slices, seed):
    """Config-2 distribution: 0.5·N(0,1) tokens, K with a per-(key block, head) offset ~ N(0, 0.3²)."""
    s = bh * bw
    nq, nk = q_slices * s, kv_slices * s
    c = heads * 128
    q = detrand.normal(seed * 10 + 0, (nq * 128, c), std=0.5)
    k = detrand.normal(seed * 10 + 1, (nk * 128, c), std=0.5)
    off = detrand.normal(seed * 10 + 2, (nk, 1, c), std=0.3, bf16_exact=False)
    k = (k.reshape(nk, 128, c) + off).reshape(nk * 128, c).astype(np.float32)
    u = k.view(np.uint32).astype(np.uint64)
    k = (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16).astype(np.uint32).view(np.float32).reshape(k.shape)
    return q, k


def local_mask(bh, bw, r):
    half = r // 2
    s = bh * bw
    m = np.zeros((s, s), bool)
    for qr in range(bh):
        for qc in range(bw):
            for kr in range(bh):
                for kc in range(bw):
                    m[qr * bw + qc, kr * bw + kc] = (qr - half <= kr <= qr - half + r - 1) and \
                                                    (qc - half <= kc <= qc - half + r - 1)
    return m


def select_f64(q, k, heads, q_slices, s, local, topk):
    """DiT.swift:158-174 in float64, one line per reference line."""
    nq, nk = q.shape[0] // 128, k.shape[0] // 128
    d = q.shape[1] // heads
    pq = q.astype(np.float64).reshape(nq, 128, -1).mean(axis=1).reshape(nq, heads, d).transpose(1, 0, 2)   # 161
    pk = k.astype(np.float64).reshape(nk, 128, -1).mean(axis=1).reshape(nk, heads, d).transpose(1, 0, 2)   # 162
    scores = np.matmul(pq, pk.transpose(0, 2, 1)) / np.sqrt(d)                                              # 163
    lm = np.where(local, 0.0, -np.inf)                                                                       # 165
    tiled = np.broadcast_to(lm.reshape(1, s, 1, s), (nq // s, s, nk // s, s)).reshape(nq, nk)                # 166
    scores = scores + tiled                                                                                  # 167
    e = np.exp(scores - scores.max(axis=-1, keepdims=True))
    attn = e / e.sum(axis=-1, keepdims=True)                                                                 # 168
    flat = attn.reshape(heads * q_slices, (nq // q_slices) * nk)                                             # 169
    n = flat.shape[1]
    kk = min(n - 1, topk)                                                                                    # 171
    thr = np.sort(flat, axis=1)[:, n - 1 - kk:n - kk]                                                        # 172
    return (flat > thr).reshape(heads, nq, nk), attn                                                         # 173


def allowed_per_row(bh, bw, q_slices, kv_slices, r):
    loc = local_mask(bh, bw, r)
    return int(loc.sum()) * kv_slices  # per (head, slice) row: each of the s query blocks × kv slices


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="the xocialize/mlx-flashvsr-swift source tree")
    args = ap.parse_args()
    spec = importlib.util.spec_from_file_location("ref_block_sparse_attn",
                                                  Path(args.reference) / "oracle" / "block_sparse_attn.py")
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    import torch
    torch.set_num_threads(1)

    for name, heads, nq, nk, density, seed, empty in ATTN_CASES:
        q, k, v, mask = attn_inputs(heads, nq, nk, density, seed, empty)
        lq, lk = nq * 128, nk * 128
        tq = torch.from_numpy(q).reshape(lq, heads, 128)
        tk = torch.from_numpy(k).reshape(lk, heads, 128)
        tv = torch.from_numpy(v).reshape(lk, heads, 128)
        bm = torch.from_numpy(mask).reshape(1, heads, nq, nk)
        out = ref.block_sparse_attn_func(tq, tk, tv, None, None, torch.ones(heads, dtype=torch.int32), None, bm,
                                         lq, lk, 0.0, softmax_scale=None)
        out = out.reshape(lq, heads * 128).numpy().astype(np.float32)
        np.savez(HERE / f"{name}.npz", mask=mask.astype(np.uint8), out=out,
                 meta=np.array([heads, nq, nk, seed, empty[0], empty[1]], np.int64),
                 density=np.array([density]))
        print(name, out.shape, "empty rows", int((mask.sum(-1) == 0).sum()))

    for name, heads, bh, bw, qs, kvs, r, keep, seed in SELECT_CASES:
        s = bh * bw
        q, k = select_inputs(heads, bh, bw, qs, kvs, seed)
        loc = local_mask(bh, bw, r)
        allowed = allowed_per_row(bh, bw, qs, kvs, r)
        topk = int(round(keep * allowed))
        mask, probs = select_f64(q, k, heads, qs, s, loc, topk)
        np.savez(HERE / f"{name}.npz", mask=mask.astype(np.uint8), probs=probs,
                 meta=np.array([heads, bh, bw, qs, kvs, r, topk, seed], np.int64))
        print(name, "topk", topk, "kept", int(mask.sum()), "of", mask.size)


if __name__ == "__main__":
    main()
