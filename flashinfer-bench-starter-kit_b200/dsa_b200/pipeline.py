"""One DSA decode step -- indexer -> sparse attention -- as CUDA graphs.

The indexer's top-2048 slot ids feed attention directly (same global slot
numbering: block_table[b, t/64]*64 + t%64 indexes the ckv / kpe caches the way
it indexes the FP8 index cache).  Every launch reads seq_lens and indices on
the device, so the whole step can be captured once and replayed for any new
lengths written into the same input buffers; the reference instead re-keys a
graph cache on the host-side seq_lens values every call
(dsa_indexer/solution/triton/kernel.py:375-384).

``DecodeStep(..., streams=2)`` splits the batch in two halves and runs
indexer(half 1) -> attention(half 1) on a side stream while indexer(half 2)
-> attention(half 2) runs on the main one, joined by events inside the graph.

``DecodeStep(..., host_io=True)`` keeps the step's per-step inputs (indexer
queries, weights, lengths, block table; attention queries) in one device
buffer and its outputs (indices, attention output, lse) in another, with a
pinned host mirror of each (``host_in`` / ``host_out``, views shaped like the
tensors).  ``replay_io()`` replays one graph that copies the inputs in, runs
the step and copies the outputs back: one launch per step on the host, for
callers whose batches are too small to hide two eager calls' host time.  The
KV caches stay resident on the device.
"""

from __future__ import annotations

import dataclasses

import torch

from . import attention, indexer, workloads


def _arena(tensors, device=None, pinned=False):
    """One byte buffer holding every tensor of `tensors` (256-byte aligned
    offsets) and views of it shaped like them."""
    offs, off = [], 0
    for t in tensors:
        offs.append(off)
        off += (t.numel() * t.element_size() + 255) // 256 * 256
    buf = torch.empty(max(off, 256), dtype=torch.uint8, device=device)
    if pinned:
        buf = buf.pin_memory()
    views = [buf[o:o + t.numel() * t.element_size()].view(t.dtype).view(t.shape)
             for o, t in zip(offs, tensors)]
    return buf, views


class DecodeStep:
    def __init__(self, dec: workloads.DecodeInputs, use_graph: bool = True, streams: int = 1,
                 host_io: bool = False):
        ix = dec.indexer
        B = ix.q_index_fp8.shape[0]
        dev = ix.q_index_fp8.device
        self.device = dev
        self.host_io = host_io and use_graph
        outs = [torch.full((B, workloads.TOPK), -1, dtype=torch.int32),
                torch.zeros(B, workloads.A_HEADS, workloads.CKV, dtype=torch.bfloat16),
                torch.zeros(B, workloads.A_HEADS, dtype=torch.float32)]
        if self.host_io:
            ins = [ix.q_index_fp8, ix.weights, ix.seq_lens, ix.block_table, dec.q_nope, dec.q_pe]
            self._in_dev, dv = _arena(ins, device=dev)
            for d, t in zip(dv, ins):
                d.copy_(t)
            self._in_host, self.host_in = _arena(ins, pinned=True)
            for h, t in zip(self.host_in, ins):
                h.copy_(t)
            dec = dataclasses.replace(
                dec, q_nope=dv[4], q_pe=dv[5],
                indexer=dataclasses.replace(ix, q_index_fp8=dv[0], weights=dv[1], seq_lens=dv[2],
                                            block_table=dv[3]))
            self._out_dev, (self.topk, self.out, self.lse) = _arena(outs, device=dev)
            for d, t in zip((self.topk, self.out, self.lse), outs):
                d.copy_(t)
            self._out_host, self.host_out = _arena(outs, pinned=True)
        else:
            self.topk, self.out, self.lse = (t.to(dev) for t in outs)
        self.dec = dec
        self.streams = max(1, min(streams, B)) if B > 0 else 1
        bounds = [B * k // self.streams for k in range(self.streams + 1)]
        self.parts = [(bounds[k], bounds[k + 1]) for k in range(self.streams)]
        self.side = [torch.cuda.Stream(dev) for _ in range(self.streams - 1)]
        # Workspaces are per stream, so warm up on the very streams the graphs
        # are captured on: nothing is allocated or moved after capture.
        self.cap = torch.cuda.Stream(dev)
        self.cap.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(self.cap):
            self.indexer_eager()
            self.attention_eager()
            self.step_eager()
        torch.cuda.synchronize(dev)
        self.g_ix = self.g_at = self.g_step = self.g_io = None
        if use_graph:
            self.g_ix = self._capture(self.indexer_eager)
            self.g_at = self._capture(self.attention_eager)
            self.g_step = self._capture(self.step_eager)
        if self.host_io:
            self.g_io = self._capture(self._io_step)

    # -- eager pieces (the public operator API) ---------------------------
    def _ix(self, lo: int, hi: int) -> None:
        ix = self.dec.indexer
        indexer.run(ix.q_index_fp8[lo:hi], ix.k_index_cache_fp8, ix.weights[lo:hi],
                    ix.seq_lens[lo:hi], ix.block_table[lo:hi], self.topk[lo:hi])

    def _at(self, lo: int, hi: int) -> None:
        d = self.dec
        attention.run(d.q_nope[lo:hi], d.q_pe[lo:hi], d.ckv_cache, d.kpe_cache,
                      self.topk[lo:hi], d.sm_scale, self.out[lo:hi], self.lse[lo:hi])

    def indexer_eager(self) -> None:
        self._ix(0, self.topk.shape[0])

    def attention_eager(self) -> None:
        self._at(0, self.topk.shape[0])

    def step_eager(self) -> None:
        if self.streams == 1:
            self._ix(0, self.topk.shape[0])
            self._at(0, self.topk.shape[0])
            return
        main = torch.cuda.current_stream(self.device)
        for s in self.side:
            s.wait_stream(main)
        for k, (lo, hi) in enumerate(self.parts):
            st = main if k == len(self.parts) - 1 else self.side[k]
            with torch.cuda.stream(st):
                self._ix(lo, hi)
                self._at(lo, hi)
        for s in self.side:
            main.wait_stream(s)

    # -- graphs -------------------------------------------------------------
    def _capture(self, fn) -> torch.cuda.CUDAGraph:
        g = torch.cuda.CUDAGraph()
        self.cap.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.cap):
            with torch.cuda.graph(g, stream=self.cap):
                fn()
        torch.cuda.current_stream(self.device).wait_stream(self.cap)
        return g

    def indexer_graph(self) -> None:
        self.g_ix.replay() if self.g_ix is not None else self.indexer_eager()

    def attention_graph(self) -> None:
        self.g_at.replay() if self.g_at is not None else self.attention_eager()

    def __call__(self) -> None:
        self.g_step.replay() if self.g_step is not None else self.step_eager()

    # -- host I/O -------------------------------------------------------------
    def _io_step(self) -> None:
        self._in_dev.copy_(self._in_host, non_blocking=True)
        self.step_eager()
        self._out_host.copy_(self._out_dev, non_blocking=True)

    def replay_io(self) -> None:
        """Copies host_in to the device, runs the step and copies the results
        into host_out, all on the current stream (one graph launch); the
        caller synchronises before reading host_out or rewriting host_in."""
        if self.g_io is None:
            raise RuntimeError("DecodeStep was built without host_io=True (and use_graph=True)")
        self.g_io.replay()
