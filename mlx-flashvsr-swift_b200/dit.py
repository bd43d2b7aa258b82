"""One FlashVSR DiT block on the B200 kernels — the host side of DiTBlock / blockForward (DiT.swift:366-381,
486-549) for one streamed chunk, each step one C-ABI call:

  inX   = norm1(tok)·(1 + scaleMSA) + shiftMSA                    fvsr_layernorm (modulated)
  q,k,v = sa.q / sa.k / sa.v (inX)                                 fvsr_linear_qkv (one tcgen05 GEMM)
  attn  = LCSA: normQ/normK, RoPE, windows, cache, selection,
          block-sparse attention, windowReverse                   fvsr_lcsa_forward_tokens (the path)
  tok   = tok + gateMSA · sa.o(attn)                               fvsr_linear, gated residual, in place
  caIn  = norm3(tok)                                               fvsr_layernorm (affine)
  cq    = normQ(ca.q(caIn))                                        fvsr_linear + fvsr_rmsnorm
  tok   = tok + ca.o(SDPA(cq, cacheK, cacheV))                     fvsr_cross_attention + fvsr_linear (gate 1)
  inF   = norm2(tok)·(1 + scaleMLP) + shiftMLP                     fvsr_layernorm (modulated)
  tok   = tok + gateMLP · ffn2(GELU(ffn1(inF)))                    fvsr_linear (GELU), fvsr_linear (gated residual)

Weights are bf16 in the nn.Linear layout (out, in); the cross-attention's context K/V are the block's cached
constants (CrossAttention.initCache, DiT.swift:346-350). The 6 modulation rows are the block's modulation plus the
step's time embedding, as the reference adds them (DiT.swift:489)."""
from __future__ import annotations

from dataclasses import dataclass

from . import (FVSR_LINEAR_GATED_RESIDUAL, FVSR_LINEAR_GELU, cross_attention, layernorm, lcsa_forward_tokens, linear,
               linear_qkv, rmsnorm)


@dataclass
class BlockWeights:
    w_qkv: object      # (3C, C): [Wq; Wk; Wv]
    b_qkv: object      # (3C)
    norm_q: object     # (C) self-attention WanRMSNorm weights
    norm_k: object
    w_o: object        # (C, C)
    b_o: object
    n3_w: object       # (C) norm3 (affine)
    n3_b: object
    ca_wq: object      # (C, C)
    ca_bq: object
    ca_norm_q: object  # (C)
    ca_wo: object      # (C, C)
    ca_bo: object
    w1: object         # (F, C)
    b1: object         # (F)
    w2: object         # (C, F)
    b2: object         # (C)
    ctx_k: object      # (Lc, C) cached cross-attention keys (normK already applied)
    ctx_v: object      # (Lc, C)

    @staticmethod
    def random(c: int = 1536, f: int = 8960, lc: int = 512, seed: int = 0, device="cuda") -> "BlockWeights":
        """Random-initialised weights of the model's shapes (no checkpoint is involved in this path)."""
        import torch
        g = torch.Generator(device=device).manual_seed(seed)

        def r(*shape, s=1.0):
            return (s * torch.randn(shape, generator=g, device=device)).to(torch.bfloat16)

        return BlockWeights(
            w_qkv=r(3 * c, c, s=c ** -0.5), b_qkv=r(3 * c, s=0.05), norm_q=(1 + r(c, s=0.1).float()).to(torch.bfloat16),
            norm_k=(1 + r(c, s=0.1).float()).to(torch.bfloat16), w_o=r(c, c, s=c ** -0.5), b_o=r(c, s=0.05),
            n3_w=(1 + r(c, s=0.1).float()).to(torch.bfloat16), n3_b=r(c, s=0.05), ca_wq=r(c, c, s=c ** -0.5),
            ca_bq=r(c, s=0.05), ca_norm_q=(1 + r(c, s=0.1).float()).to(torch.bfloat16), ca_wo=r(c, c, s=c ** -0.5),
            ca_bo=r(c, s=0.05), w1=r(f, c, s=c ** -0.5), b1=r(f, s=0.05), w2=r(c, f, s=f ** -0.5), b2=r(c, s=0.05),
            ctx_k=r(lc, c), ctx_v=r(lc, c))


class BlockBuffers:
    """Scratch of one block call for a chunk of `rows` tokens (reused across blocks and chunks)."""

    def __init__(self, rows: int, c: int, f: int, device="cuda"):
        import torch

        def e(n):
            return torch.empty((rows, n), dtype=torch.bfloat16, device=device)

        self.inx, self.q, self.k, self.v, self.qwin, self.attn = (e(c) for _ in range(6))
        self.cq_lin, self.cq, self.ca = e(c), e(c), e(c)
        self.h = e(f)
        self.ones = torch.ones((c,), dtype=torch.bfloat16, device=device)


def block_forward(w: BlockWeights, tok, mod6, cache, geom, rope, buf: BlockBuffers, workspace, eps: float = 1e-6,
                  kidx=None, kcnt=None, stream=None, timeline=None):
    """blockForward (DiT.swift:486-549) for one chunk: tok (L, C) bf16 token order, updated in place and returned;
    mod6 = (shiftMSA, scaleMSA, gateMSA, shiftMLP, scaleMLP, gateMLP), each (C) bf16; cache = the block's window K/V
    cache (KVCache); geom = the chunk's LCSA geometry; rope = the chunk's (cos, sin) tables. timeline: optional list
    that receives (stage, CUDA event recorded after it) for a per-stage breakdown."""
    import torch
    st = stream if stream is not None else torch.cuda.current_stream()

    def mark(name):
        if timeline is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(st)
            timeline.append((name, ev))

    mark("begin")
    shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = mod6
    heads = geom.heads
    layernorm(tok, shift=shift_msa, scale=scale_msa, eps=eps, out=buf.inx, stream=stream)
    mark("norm1")
    linear_qkv(buf.inx, w.w_qkv, w.b_qkv, outs=(buf.q, buf.k, buf.v), stream=stream)
    mark("qkv")
    lcsa_forward_tokens(buf.q, buf.k, buf.v, cache, geom, norm_q=w.norm_q, norm_k=w.norm_k, eps=eps, rope=rope,
                        q_win=buf.qwin, out=buf.attn, kidx=kidx, kcnt=kcnt, workspace=workspace, stream=stream)
    mark("lcsa")
    linear(buf.attn, w.w_o, w.b_o, epilogue=FVSR_LINEAR_GATED_RESIDUAL, gate=gate_msa, resid=tok, out=tok,
           stream=stream)
    mark("o")
    layernorm(tok, weight=w.n3_w, bias=w.n3_b, eps=eps, out=buf.inx, stream=stream)
    mark("norm3")
    linear(buf.inx, w.ca_wq, w.ca_bq, out=buf.cq_lin, stream=stream)
    mark("ca.q")
    rmsnorm(buf.cq_lin, w.ca_norm_q, eps=eps, out=buf.cq, stream=stream)
    mark("ca.norm_q")
    cross_attention(buf.cq, w.ctx_k, w.ctx_v, heads, out=buf.ca, stream=stream)
    mark("ca.attention")
    linear(buf.ca, w.ca_wo, w.ca_bo, epilogue=FVSR_LINEAR_GATED_RESIDUAL, gate=buf.ones, resid=tok, out=tok,
           stream=stream)
    mark("ca.o")
    layernorm(tok, shift=shift_mlp, scale=scale_mlp, eps=eps, out=buf.inx, stream=stream)
    mark("norm2")
    linear(buf.inx, w.w1, w.b1, epilogue=FVSR_LINEAR_GELU, out=buf.h, stream=stream)
    mark("ffn1 (GELU)")
    linear(buf.h, w.w2, w.b2, epilogue=FVSR_LINEAR_GATED_RESIDUAL, gate=gate_mlp, resid=tok, out=tok,
           stream=stream)
    mark("ffn2")
    return tok


def block_flops(rows: int, c: int, f: int, lc: int, kept_triples: int) -> float:
    """Algorithmic FLOPs of one block call: the six linear layers (2·rows·in·out each), the LCSA over its kept
    (head, query block, key block) triples (4·128³ each) and the dense cross-attention (4·128 per query × context key
    × head, i.e. 4·rows·lc·c)."""
    linears = 2.0 * rows * c * (3 * c + c + c + c + f) + 2.0 * rows * f * c
    lcsa = 4.0 * 128 ** 3 * kept_triples
    cross = 4.0 * rows * lc * c
    return linears + lcsa + cross
