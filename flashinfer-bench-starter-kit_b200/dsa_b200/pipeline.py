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
"""

from __future__ import annotations

import torch

from . import attention, indexer, workloads


class DecodeStep:
    def __init__(self, dec: workloads.DecodeInputs, use_graph: bool = True, streams: int = 1):
        self.dec = dec
        ix = dec.indexer
        B = ix.q_index_fp8.shape[0]
        dev = ix.q_index_fp8.device
        self.device = dev
        self.topk = torch.full((B, workloads.TOPK), -1, dtype=torch.int32, device=dev)
        self.out = torch.zeros(B, workloads.A_HEADS, workloads.CKV, dtype=torch.bfloat16, device=dev)
        self.lse = torch.zeros(B, workloads.A_HEADS, dtype=torch.float32, device=dev)
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
        self.g_ix = self.g_at = self.g_step = None
        if use_graph:
            self.g_ix = self._capture(self.indexer_eager)
            self.g_at = self._capture(self.attention_eager)
            self.g_step = self._capture(self.step_eager)

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
