"""GPU parity of one whole DiT block (blockForward, DiT.swift:486-549) assembled from the library's C-ABI calls
(dit.block_forward): two streamed chunks through one block and its window K/V cache, against an fp32 restatement of
the block in torch whose LCSA core is the oracle's (WanRMSNorm + RoPE + windowPartition, attention over the kept
blocks, windowReverse). The reference is fed the library's own selection (kidx/kcnt; the selection itself is checked
bit for bit elsewhere) and rounds to bf16 at the points where the library stores bf16.

Tolerance: rel = max|got − ref| / max|ref| ≤ 1e-2 for every stage compared (the attention cores round P to bf16 and
each layer stores bf16), and ≤ 2e-2 on the block's update (out − in)."""
from __future__ import annotations

import importlib

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

REL = 1e-2
REL_UPDATE = 2e-2


@pytest.fixture(scope="module")
def dev(fvsr):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return "cuda"


def bits(t):
    return t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def bf(t):
    return t.to(torch.bfloat16)


def rel(got, ref):
    got, ref = got.double(), ref.double()
    return ((got - ref).abs().max() / ref.abs().max().clamp_min(1e-30)).item()


class RefBlock:
    """The block in fp32 torch (plus the oracle's LCSA core) with bf16 rounding at the library's storage points."""

    def __init__(self, orc, w, heads, kv_len, eps=1e-6):
        self.orc, self.w, self.heads, self.kv_len, self.eps = orc, w, heads, kv_len, eps
        self.cache_k, self.cache_v = [], []   # per slice: window-order bf16 bits

    def ln(self, x, weight=None, bias=None):
        c = x.shape[-1]
        return torch.nn.functional.layer_norm(x.float(), (c,), None if weight is None else weight.float(),
                                              None if bias is None else bias.float(), eps=self.eps)

    @staticmethod
    def lin(x, wt, b):
        return x.float() @ wt.float().t() + b.float()

    def __call__(self, tok, mod6, kidx, kcnt, rope, f, h, w):
        orc, W, H, eps = self.orc, self.w, self.heads, self.eps
        c = tok.shape[1]
        sh1, sc1, g1, sh2, sc2, g2 = (m.float() for m in mod6)
        inx = bf(self.ln(tok) * (1 + sc1) + sh1)
        q, k, v = (bf(self.lin(inx, W.w_qkv[i * c:(i + 1) * c], W.b_qkv[i * c:(i + 1) * c])) for i in range(3))
        cos, sin = (t.cpu().numpy() for t in rope)
        qw = orc.prepare(bits(q), f, h, w, H, weight=bits(W.norm_q), eps=eps, cos=cos, sin=sin)
        kw = orc.prepare(bits(k), f, h, w, H, weight=bits(W.norm_k), eps=eps, cos=cos, sin=sin)
        vw = orc.prepare(bits(v), f, h, w, H)
        per = kw.shape[0] // (f // 2)          # rows of one temporal slice
        new_k = [kw[i * per:(i + 1) * per] for i in range(f // 2)]
        new_v = [vw[i * per:(i + 1) * per] for i in range(f // 2)]
        kcat = np.concatenate(self.cache_k + new_k)
        vcat = np.concatenate(self.cache_v + new_v)
        f32 = orc.bf16_bits_to_f32
        att = orc.attention(f32(qw), f32(kcat), f32(vcat), kidx.cpu().numpy(), kcnt.cpu().numpy(), H)
        attn = bf(torch.from_numpy(orc.window_reverse(att, 1, f, h, w).reshape(tok.shape)).to(tok.device))
        # DiT.swift:532-538: keep the cache ⊕ current, dropping the oldest slice once if more than kvLen are held
        self.cache_k, self.cache_v = self.cache_k + new_k, self.cache_v + new_v
        if len(self.cache_k) > self.kv_len:
            self.cache_k, self.cache_v = self.cache_k[1:], self.cache_v[1:]
        tok1 = bf(tok.float() + g1 * self.lin(attn, W.w_o, W.b_o))
        n3 = bf(self.ln(tok1, W.n3_w, W.n3_b))
        cql = self.lin(n3, W.ca_wq, W.ca_bq).to(torch.bfloat16).float()
        cq = bf(bf(cql * torch.rsqrt((cql * cql).mean(-1, keepdim=True) + eps)).float() * W.ca_norm_q.float())
        L, Lc = cq.shape[0], W.ctx_k.shape[0]
        qh = cq.float().view(L, H, 128).transpose(0, 1)
        kh = W.ctx_k.float().view(Lc, H, 128).transpose(0, 1)
        vh = W.ctx_v.float().view(Lc, H, 128).transpose(0, 1)
        ca = bf(torch.softmax(qh @ kh.transpose(1, 2) / 128 ** 0.5, dim=-1) @ vh).transpose(0, 1).reshape(L, c)
        tok2 = bf(tok1.float() + self.lin(ca, W.ca_wo, W.ca_bo))
        inf = bf(self.ln(tok2) * (1 + sc2) + sh2)
        hid = bf(torch.nn.functional.gelu(self.lin(inf, W.w1, W.b1), approximate="tanh"))
        out = bf(tok2.float() + g2 * self.lin(hid, W.w2, W.b2))
        return {"attn": attn, "ca": ca, "hid": hid, "out": out}


def test_block_two_chunks_against_reference(fvsr, orc, dev):
    dit = importlib.import_module("fvsr_b200.dit")
    heads, bh, bw, kv_len, ffn, lc = 2, 3, 5, 2, 512, 256
    c = heads * 128
    w = dit.BlockWeights.random(c=c, f=ffn, lc=lc, seed=11)
    g0 = fvsr.Geometry(heads=heads, bh=bh, bw=bw, q_slices=2, kv_slices=2, local_range=11, dtype=fvsr.FVSR_BF16)
    cache = fvsr.KVCache(g0, kv_len=kv_len, max_new_slices=2)
    ref = RefBlock(orc, w, heads, kv_len)
    gen = torch.Generator(device="cuda").manual_seed(77)
    held = 0
    for chunk, qs in enumerate((2, 1)):
        kv_total = min(held + qs, kv_len + 1)
        g = fvsr.Geometry(**{**g0.__dict__, "q_slices": qs})
        gfull = fvsr.Geometry(**{**g.__dict__, "kv_slices": kv_total})
        g.topk = gfull.topk = int(round(0.5 * gfull.allowed_per_row()))
        rows = g.nq * 128
        f, h, ww = 2 * qs, 8 * bh, 8 * bw
        tok = torch.randn((rows, c), generator=gen, device="cuda").to(torch.bfloat16)
        mod6 = [(s * torch.randn((c,), generator=gen, device="cuda")).to(torch.bfloat16)
                for s in (0.2, 0.2, 0.5, 0.2, 0.2, 0.5)]
        rope = fvsr.rope_tables(f, h, ww, t0=0 if chunk == 0 else 4)
        kidx = torch.empty((heads, gfull.nq, gfull.nk), dtype=torch.int32, device="cuda")
        kcnt = torch.empty((heads, gfull.nq), dtype=torch.int32, device="cuda")
        buf = dit.BlockBuffers(rows, c, ffn)
        tok_in = tok.clone()
        got = dit.block_forward(w, tok, mod6, cache, g, rope, buf, fvsr.make_workspace(gfull), kidx=kidx, kcnt=kcnt)
        torch.cuda.synchronize()
        assert got.data_ptr() == tok.data_ptr()
        want = ref(tok_in, mod6, kidx, kcnt, rope, f, h, ww)
        for name, mine in (("attn", buf.attn), ("ca", buf.ca), ("hid", buf.h), ("out", got)):
            r = rel(mine, want[name])
            assert r <= REL, f"chunk {chunk} {name}: rel {r:.3e}"
        r = rel(got.float() - tok_in.float(), want["out"].float() - tok_in.float())
        assert r <= REL_UPDATE, f"chunk {chunk} update: rel {r:.3e}"
        held = min(held + qs, kv_len) if chunk else qs
        assert cache.slices == held
    cache.close()
    fvsr.device_check()

