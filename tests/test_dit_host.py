"""Host side of the DiT block module (dit.py), no GPU: the weights' shapes follow the model's Linear layout
(DiT.swift:330-381) and the FLOP count covers every layer of blockForward (DiT.swift:486-549)."""
from __future__ import annotations

import importlib

import pytest

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def dit():
    from conftest import load_product
    load_product()
    return importlib.import_module("fvsr_b200.dit")


def test_block_weights_shapes(dit):
    c, f, lc = 256, 512, 128
    w = dit.BlockWeights.random(c=c, f=f, lc=lc, seed=1, device="cpu")
    want = {"w_qkv": (3 * c, c), "b_qkv": (3 * c,), "w_o": (c, c), "ca_wq": (c, c), "ca_wo": (c, c), "w1": (f, c),
            "b1": (f,), "w2": (c, f), "b2": (c,), "ctx_k": (lc, c), "ctx_v": (lc, c), "norm_q": (c,), "n3_b": (c,)}
    for name, shape in want.items():
        t = getattr(w, name)
        assert tuple(t.shape) == shape, name
        assert t.dtype == torch.bfloat16, name


def test_block_flops_counts_every_layer(dit):
    rows, c, f, lc, kept = 256, 256, 512, 128, 3
    linears = 2 * rows * c * (3 * c) + 3 * (2 * rows * c * c) + 2 * rows * c * f + 2 * rows * f * c
    want = linears + 4 * 128 ** 3 * kept + 4 * rows * lc * c
    assert dit.block_flops(rows, c, f, lc, kept) == want
