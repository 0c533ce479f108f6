"""The reference's own GPU solutions, run on the GPU (TEST INFRASTRUCTURE ONLY).

``oracle/build_ref.py`` compiles the reference's inline CUDA/C++ sources,
unmodified, into ``oracle/_ref/dsa_topk_s11.so`` and ``dsa_sparse_v8.so``.
This module loads them and restates the two Python ``run()`` wrappers around
them, so that the reference's stock code path can serve for a parity check
and as the same-box GPU baseline:

* ``RefIndexer.run`` follows dsa_indexer/solution/triton/kernel.py:364-436:
  ``.contiguous()`` on the inputs, a host copy of ``seq_lens`` (a device
  sync) that keys a graph cache together with the shapes, three eager calls
  of ``dsa_topk_run_ms`` per key, then one CUDA-graph capture over static
  input buffers, and afterwards copy-in -> replay -> copy-out on every call.
* ``ref_attention_run`` follows dsa_attention/solution/triton/kernel.py:240-252:
  flatten the caches to ``[-1, 512]`` / ``[-1, 64]``, cast the indices to
  int32 and call ``dsa_sparse_attention`` with TOPK = 2048 (no graph).

Known behaviour of the reference kept as is: an attention row whose indices
are all -1 gives NaN (its softmax divides 0 by 0); ties in the indexer are
ordered by ``at::topk``.
"""

from __future__ import annotations

import importlib.machinery
import importlib.util
import pathlib

import torch

REF_DIR = pathlib.Path(__file__).resolve().parent / "_ref"
INDEXER_SO = REF_DIR / "dsa_topk_s11.so"
ATTENTION_SO = REF_DIR / "dsa_sparse_v8.so"
WARMUP_CALLS = 3          # dsa_indexer/solution/triton/kernel.py:44
TOPK = 2048               # dsa_attention/solution/triton/kernel.py:14

_mods = {}


def available() -> bool:
    return INDEXER_SO.exists() and ATTENTION_SO.exists()


def _load(name: str, path: pathlib.Path):
    if name not in _mods:
        loader = importlib.machinery.ExtensionFileLoader(name, str(path))
        spec = importlib.util.spec_from_loader(name, loader)
        mod = importlib.util.module_from_spec(spec)
        loader.exec_module(mod)
        _mods[name] = mod
    return _mods[name]


def indexer_module():
    return _load("dsa_topk_s11", INDEXER_SO)


def attention_module():
    return _load("dsa_sparse_v8", ATTENTION_SO)


class RefIndexer:
    """The reference's indexer ``run()`` with its per-process graph cache."""

    def __init__(self):
        self.mod = indexer_module()
        self.calls = {}
        self.bufs = {}
        self.graphs = {}

    def run(self, q_index_fp8, k_index_cache_fp8, weights, seq_lens, block_table, topk_indices):
        q_c, k_c = q_index_fp8.contiguous(), k_index_cache_fp8.contiguous()
        w_c, bt_c = weights.contiguous(), block_table.contiguous()
        sl_cpu = seq_lens.cpu()                         # kernel.py:375 (device sync)
        key = (tuple(q_c.shape), tuple(k_c.shape), tuple(bt_c.shape), tuple(sl_cpu.tolist()))
        count = self.calls.get(key, 0)
        self.calls[key] = count + 1
        if key not in self.graphs:
            if key not in self.bufs:
                self.bufs[key] = {"q": torch.empty_like(q_c), "k": torch.empty_like(k_c),
                                  "w": torch.empty_like(w_c), "bt": torch.empty_like(bt_c),
                                  "out": torch.empty_like(topk_indices), "sl": sl_cpu.clone()}
            sb = self.bufs[key]
            if count < WARMUP_CALLS:                    # kernel.py:397-402
                self.mod.dsa_topk_run_ms(q_c, k_c, w_c, sl_cpu, bt_c, topk_indices)
            else:                                       # kernel.py:404-423
                sb["q"].copy_(q_c)
                sb["k"].copy_(k_c)
                sb["w"].copy_(w_c)
                sb["bt"].copy_(bt_c)
                torch.cuda.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    self.mod.dsa_topk_run_ms(sb["q"], sb["k"], sb["w"], sb["sl"], sb["bt"], sb["out"])
                self.graphs[key] = g
                g.replay()
                topk_indices.copy_(sb["out"])
        else:                                           # kernel.py:425-436
            sb = self.bufs[key]
            sb["q"].copy_(q_c, non_blocking=True)
            sb["k"].copy_(k_c, non_blocking=True)
            sb["w"].copy_(w_c, non_blocking=True)
            sb["bt"].copy_(bt_c, non_blocking=True)
            self.graphs[key].replay()
            topk_indices.copy_(sb["out"], non_blocking=True)

    def replay_only(self, seq_lens_key: tuple, q_shape, k_shape, bt_shape) -> None:
        """Replays the captured graph of a key without the static-buffer
        copies around it (for a kernel-only timing next to the stock path)."""
        self.graphs[(tuple(q_shape), tuple(k_shape), tuple(bt_shape), seq_lens_key)].replay()


@torch.no_grad()
def ref_attention_run(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, sm_scale, output, lse):
    mod = attention_module()
    num_tokens = q_nope.shape[0]
    ckv_flat = ckv_cache.reshape(-1, 512)
    kpe_flat = kpe_cache.reshape(-1, 64)
    idx = sparse_indices.int() if sparse_indices.dtype != torch.int32 else sparse_indices
    mod.dsa_sparse_attention(ckv_flat, kpe_flat, q_nope, q_pe, idx, sm_scale, output, lse,
                             num_tokens, TOPK)
