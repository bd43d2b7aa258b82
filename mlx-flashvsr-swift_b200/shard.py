"""The query-block partition of one streamed chunk over the GPUs of a node (one process per GPU).

Rank r holds the chunk's query blocks (windows) of its shard — q, k_new and v_new rows as a sequence-split QKV
projection leaves them — and, per DiT layer, a replica of that layer's window cache. One layer call
(`ShardedChunk.layer`), per the reference's blockForward (DiT.swift:504-538) split over ranks:
  1. pool the rank's q and k_new shards (fvsr_lcsa_pool: the fp32 block means of DiT.swift:161-162);
  2. all-gather the pooled rows of every rank: the queries into one (Nq, H·128) buffer, the keys straight into the
     cache page reserved for the current slice — on the compute stream (1.7 MB at config 3);
  3. all-gather the current slice's K and V shards straight into that page on a high-priority communication stream
     (106 MB at config 3, 189 MB at config 5) — the concat of DiT.swift:508-511 without a copy — beside
  4. fvsr_lcsa_select_shard: the full selection over the gathered pooled rows (every rank computes the same one); its
     cooperative launch leaves `spare_sms` SMs to the gather's kernel (with spare_sms = 0 it needs every SM, and the
     gather is issued after it instead), and
  5. fvsr_lcsa_attend_shard: the attention of the rank's query blocks over every head — first the kept blocks in
     the cached slices (fp32 partials), then, once the gather has landed, the current slice's blocks, merged — and
     the trim.
The gathers write equal padded shards of ceil(Nq / N) blocks, so the cache pages are ceil(Nq / N)·N blocks long.
At N = 1 the same call is fvsr_lcsa_forward (append, select, attend, trim) with no collective.
"""
from __future__ import annotations

import ctypes


class ShardedChunk:
    """Per-rank state of the partition for `layers` DiT layers of one chunk geometry (q_slices = 1: a steady chunk)."""

    def __init__(self, pkg, geom, kv_len: int, layers: int, rank: int, world: int, comm=None, device=None,
                 split: bool = True, spare_sms: int = 32):
        import torch
        if geom.q_slices != 1:
            raise pkg.FVSRError(pkg.FVSR_EINVAL, "the sharded chunk takes one temporal slice per chunk")
        if world > 1 and comm is None:
            raise pkg.FVSRError(pkg.FVSR_EINVAL, "world > 1 needs a communicator")
        self.pkg, self.geom, self.kv_len, self.layers = pkg, geom, kv_len, layers
        self.rank, self.world, self.comm = rank, world, comm
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.shard = pkg.query_shard(geom.nq, world, rank)
        w = self.shard.width
        self.page_blocks = max(geom.s, w * world)
        self.caches = [pkg.KVCache(geom, kv_len, 1, self.page_blocks) for _ in range(layers)]
        c = geom.channels
        self.pq_send = torch.zeros((w, c), dtype=torch.float32, device=self.device)
        self.pk_send = torch.zeros((w, c), dtype=torch.float32, device=self.device)
        self.pq_full = torch.zeros((w * world, c), dtype=torch.float32, device=self.device)
        self.full = pkg.Geometry(**{**geom.__dict__, "kv_slices": kv_len + 1})
        self.workspace = pkg.make_workspace(self.full, self.device)
        self.partial = (torch.empty(pkg.partial_size(geom, self.shard), dtype=torch.uint8, device=self.device)
                        if split and geom.dtype == pkg.FVSR_BF16 and self.shard.blocks else None)
        # the gathers' stream outranks the compute stream, so NCCL's CTAs take the next SMs the attention frees instead
        # of queueing behind the whole first-part grid
        self.comm_stream = torch.cuda.Stream(device=self.device, priority=-1)
        self.kv_ready = [torch.cuda.Event() for _ in range(2)]
        self.spare_sms = spare_sms
        self.calls = 0

    def shard_rows(self) -> int:
        """Token rows of the padded shard buffers k_new / v_new must have (width·128)."""
        return self.shard.width * 128

    def prefill(self, layer: int, k_slices, v_slices) -> None:
        """Puts kv_len whole slices (each (s·128, H·128), oldest first) into a layer's cache — the replicated state
        the previous chunks left on every rank."""
        for k, v in zip(k_slices, v_slices):
            self.caches[layer].append(k, v, 1)

    def layer(self, layer: int, q, k_new, v_new, out, kcnt=None, stream=None):
        """One layer call of this rank. q / out: (blocks·128, H·128); k_new / v_new: (width·128, H·128), rows past
        blocks·128 being padding. kcnt: optional (H, Nq) output. Enqueued on `stream` (default: the current one)."""
        import torch
        pkg, g, sh = self.pkg, self.geom, self.shard
        st = stream or torch.cuda.current_stream(self.device)
        cache = self.caches[layer]
        if self.world == 1:
            pkg.lcsa_forward(q, k_new[: sh.blocks * 128], v_new[: sh.blocks * 128], cache, g, out=out, kcnt=kcnt,
                             workspace=self.workspace, stream=st)
            return out
        L = pkg.lib()
        k_page, v_page, pk_page = cache.reserve()
        p = g.params()
        pkg._check(L.fvsr_lcsa_pool(ctypes.byref(p), pkg._ptr(q), sh.blocks, pkg._ptr(self.pq_send),
                                    pkg._stream(st)))
        pkg._check(L.fvsr_lcsa_pool(ctypes.byref(p), pkg._ptr(k_new), sh.blocks, pkg._ptr(self.pk_send),
                                    pkg._stream(st)))
        # pooled rows: small, on the compute stream (the selection needs them first)
        self.comm.group_start()
        self.comm.all_gather(self.pq_send, self.pq_full, st)
        self.comm.all_gather(self.pk_send, pk_page, st)
        self.comm.group_end()
        cache.commit()
        ev = self.kv_ready[self.calls & 1]
        self.calls += 1

        def kv_gather():  # after every earlier use of this page (and the pooled gather) on the compute stream
            self.comm_stream.wait_stream(st)
            self.comm.group_start()
            self.comm.all_gather(k_new, k_page, self.comm_stream)
            self.comm.all_gather(v_new, v_page, self.comm_stream)
            self.comm.group_end()
            ev.record(self.comm_stream)

        if self.spare_sms > 0:
            kv_gather()
        pkg.lcsa_select_shard(self.pq_full, sh, cache, g, self.workspace, kcnt=kcnt, spare_sms=self.spare_sms,
                              stream=st)
        if self.spare_sms <= 0:
            kv_gather()
        pkg.lcsa_attend_shard(q, sh, cache, g, self.workspace, out, kv_ready=ev, partial=self.partial, kcnt=kcnt,
                              stream=st)
        return out

    def close(self) -> None:
        for c in self.caches:
            c.close()
