"""The five benchmark/parity configurations of the LCSA path and their seeded synthetic inputs.

Geometry follows the reference's streaming DiT (Sources/FlashVSRMLX/DiT.swift:478-485, 504-538): 12 heads of 128,
128-token windows (2 latent frames × 8 × 8 patches), s = bh·bw spatial blocks per temporal slice, Nq = q_slices·s,
Nk = kv_slices·s, locality range R (default 11, Pipeline.swift:23), and an integer top-k = round(keep · allowed),
where `allowed` counts the locality-allowed (query block, key block) pairs of one (head, slice) selection row.

Inputs are synthetic (no clips or checkpoints are involved in this path): seeded normal tensors in window order,
seed = 1000·config + 30·chunk + layer.
  "normal": q, k, v ~ N(0, 1).
  "c2":     q, k, v ~ 0.5·N(0, 1), and k carries a per-(key block, head) offset vector ~ N(0, 0.3²) added to all 128
            tokens of the block, so the pooled block scores are well separated.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class Config:
    name: str
    bh: int
    bw: int
    q_slices: int
    kv_slices: int
    local_range: int
    keep: float
    dtype: str          # "f32" | "bf16"
    dist: str           # "normal" | "c2"
    heads: int = 12
    layers: int = 30

    def geometry(self, kv_slices: int | None = None, q_slices: int | None = None):
        from . import FVSR_BF16, FVSR_F32, Geometry
        g = Geometry(heads=self.heads, bh=self.bh, bw=self.bw, q_slices=q_slices or self.q_slices,
                     kv_slices=kv_slices or self.kv_slices, local_range=self.local_range,
                     dtype=FVSR_BF16 if self.dtype == "bf16" else FVSR_F32)
        g.topk = int(round(self.keep * g.allowed_per_row()))
        return g


CONFIGS = {
    1: Config("512x256 fp32, 8x24 blocks, all allowed, keep 50%", 4, 2, 1, 3, 11, 0.5, "f32", "normal"),
    2: Config("1280x768 bf16, 60x180 blocks, R=11, keep 60%", 6, 10, 1, 3, 11, 0.6, "bf16", "c2"),
    3: Config("1920x1152 bf16, 135x405 blocks, R=11, keep 30%", 9, 15, 1, 3, 11, 0.3, "bf16", "normal"),
    4: Config("1280x768 bf16 streaming, 10 chunks, kvLen 2", 6, 10, 3, 3, 11, 0.6, "bf16", "c2"),
    5: Config("2560x1536 bf16, 240x720 blocks, R=11, keep 25%", 12, 20, 1, 3, 11, 0.25, "bf16", "c2"),
}


def seed_of(config: int, chunk: int, layer: int) -> int:
    return 1000 * config + 30 * chunk + layer


def synth_qkv(cfg: Config, geom, seed: int, device="cuda", kv_rows: int | None = None):
    """Seeded (q, k, v) for one layer call: q (Nq·128, H·128), k / v (kv_rows or Nk·128, H·128), window order."""
    import torch
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    c = geom.channels
    lq = geom.nq * 128
    lk = kv_rows if kv_rows is not None else geom.nk * 128
    dt = torch.bfloat16 if cfg.dtype == "bf16" else torch.float32
    std = 0.5 if cfg.dist == "c2" else 1.0
    q = torch.randn((lq, c), generator=gen, device=device, dtype=torch.float32).mul_(std)
    k = torch.randn((lk, c), generator=gen, device=device, dtype=torch.float32).mul_(std)
    v = torch.randn((lk, c), generator=gen, device=device, dtype=torch.float32).mul_(std)
    if cfg.dist == "c2":
        off = torch.randn((lk // 128, 1, c), generator=gen, device=device, dtype=torch.float32).mul_(0.3)
        k = (k.view(lk // 128, 128, c) + off).view(lk, c)
    return q.to(dt).contiguous(), k.to(dt).contiguous(), v.to(dt).contiguous()


def kept_flops(kcnt_sum: int) -> float:
    """Algorithmic FLOPs of the attention: 4·128³ per kept (query block, key block, head) triple."""
    return 4.0 * 128 ** 3 * kcnt_sum
