"""The product's host-side rotation tables (RopeTables, DiT.swift:52-97) against the definition, on the CPU."""
from __future__ import annotations

import math

import pytest

torch = pytest.importorskip("torch")


def test_rope_tables_follow_the_grid_definition():
    from conftest import load_product
    fvsr = load_product()
    f, h, w, t0 = 4, 16, 8, 6
    cos, sin = fvsr.rope_tables(f, h, w, t0=t0, device="cpu")
    assert cos.shape == (f * h * w, 64) and sin.shape == (f * h * w, 64) and cos.dtype == torch.float32
    # entries 0..21: temporal axis (sub-dimension 44, position t0 + t); 22..42: height (42, y); 43..63: width (42, x)
    for t, y, x in [(0, 0, 0), (3, 15, 7), (2, 5, 3), (1, 9, 0)]:
        tok = (t * h + y) * w + x
        for j in range(64):
            if j < 22:
                dim, pos, jj = 44, t0 + t, j
            elif j < 43:
                dim, pos, jj = 42, y, j - 22
            else:
                dim, pos, jj = 42, x, j - 43
            a = pos * (1.0 / math.pow(10000.0, 2.0 * jj / dim))
            assert abs(cos[tok, j].item() - math.cos(a)) <= 1e-7
            assert abs(sin[tok, j].item() - math.sin(a)) <= 1e-7


def test_rope_tables_reject_positions_past_the_table_end():
    from conftest import load_product
    fvsr = load_product()
    with pytest.raises(fvsr.FVSRError):
        fvsr.rope_tables(4, 8, 8, t0=1021, device="cpu")
