"""Vocab-sharded decode tail over a torch.distributed process group.

One process per GPU; rank r owns the contiguous vocab rows
[r*V/N, (r+1)*V/N) of the int8 LM head (lal_tail_config.shard_rank/count).
A step is

  1. lal_tail_shard_select   every rank streams its slice once, applies the
                              penalty to its rows and writes per stream the
                              tie-complete local top-k record;
  2. all-gather               the records (a few hundred bytes per stream and
                              a bitmap of the slice's rows, which only a
                              record in its wide form fills) in rank order,
                              on the tail's own CUDA stream;
  3. lal_tail_shard_merge     every rank merges the same records and draws the
                              same token, pushing it into its history copy.

The reference samples in one process (runtime/lal_sampling.h:46-125); the
sharded step returns the unsharded result bit for bit because every global
candidate {l >= T} is in its slice's record and the records concatenate in
ascending vocab order.  torch is used only to move the records (NCCL on GPUs).
"""
from __future__ import annotations

from typing import Optional

import numpy as np

from . import DecodeTail, LAL_SAMPLER_LIBRARY


class _DeviceBytes:
    """A raw device range seen as a uint8 array (CUDA array interface)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1",
                                         "data": (ptr, False), "version": 3, "strides": None}


def shard_rows(vocab: int, rank: int, count: int):
    """(first row, row count) of rank's slice, as lal_tail_create computes it."""
    r0 = rank * vocab // count
    return r0, (rank + 1) * vocab // count - r0


class ShardedDecodeTail:
    """DecodeTail for this rank's slice + the record exchange.

    group: a torch.distributed process group (None = the default group);
    its backend must move CUDA tensors (NCCL).  p2p: connect the ranks'
    exchange buffers (CUDA IPC over NVLink) so that a single-stream step is
    one kernel per rank (lal_tail_connect_peers); batched steps use the
    all-gather."""

    def __init__(self, vocab_size: int, n_embd: int, device: int, max_streams: int = 1,
                 max_top_k: int = 64, history_cap: int = 256,
                 sampler: int = LAL_SAMPLER_LIBRARY, group=None, p2p: bool = True):
        import torch
        import torch.distributed as dist

        self.torch, self.dist, self.group = torch, dist, group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = device
        self.tail = DecodeTail(vocab_size, n_embd, max_streams=max_streams,
                               max_top_k=max_top_k, history_cap=history_cap, sampler=sampler,
                               device=device, shard_rank=self.rank, shard_count=self.world)
        self.torch_stream = torch.cuda.ExternalStream(self.tail.stream(), device=device)
        self._views = {}
        self.p2p = False
        if p2p:
            # exchange_handle clears this rank's receive buffer before its
            # handle leaves the rank; the gather orders every clear before
            # any rank's first step, and the barrier keeps a rank from
            # stepping before every peer has opened its mappings
            handles = [None] * self.world
            dist.all_gather_object(handles, self.tail.exchange_handle(), group=group)
            self.tail.connect_peers(handles)
            dist.barrier(group=group)
            self.p2p = True

    # the slice and the per-stream state live in the wrapped context
    def __getattr__(self, name):
        if name == "tail":
            raise AttributeError(name)
        return getattr(self.tail, name)

    def _exchange_views(self, n: int):
        v = self._views.get(n)
        if v is None:
            send, recv, nbytes = self.tail.exchange_buffers(n)
            t = self.torch
            with t.cuda.device(self.device):
                vs = t.as_tensor(_DeviceBytes(send, nbytes), device=f"cuda:{self.device}")
                vr = t.as_tensor(_DeviceBytes(recv, nbytes * self.world),
                                 device=f"cuda:{self.device}")
            v = self._views[n] = (vs, vr)
        return v

    def step_device(self, d_hidden: int, n_streams: int, d_u: int, d_tokens: int):
        """Enqueue one sharded step on the tail's stream (no host wait)."""
        if self.p2p and n_streams == 1:
            self.tail.step_device(d_hidden, n_streams, d_u, d_tokens)
            return
        self.tail.shard_select(d_hidden, n_streams)
        vs, vr = self._exchange_views(n_streams)
        with self.torch.cuda.stream(self.torch_stream):
            self.dist.all_gather_into_tensor(vr, vs, group=self.group)
        self.tail.shard_merge(n_streams, d_u, d_tokens)

    def step(self, hidden: np.ndarray, u: np.ndarray) -> np.ndarray:
        """One step from host buffers: the same tokens on every rank."""
        hidden = np.asarray(hidden)
        if self.p2p and (hidden.ndim == 1 or hidden.shape[0] == 1):
            return self.tail.step(hidden, u)
        n = self.tail.stage_inputs(hidden, u)
        d_hid, d_u, d_tok = self.tail.device_buffers()
        self.step_device(d_hid, n, d_u, d_tok)
        return self.tail.fetch_tokens(n)

    def close(self):
        """Collective: every rank's kernels finish before any buffer is freed."""
        self.tail.sync()
        self.dist.barrier(group=self.group)
        self._views.clear()
        self.tail.close()


def merge_records_host(records, vocab: int, temperature: float, top_k: int,
                       variant: int, u: float, sample_fn) -> dict:
    """Host restatement of the merge, for tests: records = [(values, indices)]
    in rank order.  The concatenated candidates are scattered into a vocab
    array of -inf and sampled by sample_fn (the reference sampler), which then
    sees exactly the gathered candidates."""
    logits = np.full(vocab, -np.inf, np.float32)
    for vals, idx in records:
        logits[np.asarray(idx, np.int64)] = vals
    return sample_fn(logits, temperature, top_k, variant, u)


def local_record(logits_slice: np.ndarray, row0: int, vocab: int, top_k: int,
                 greedy: bool) -> Optional[tuple]:
    """The record a slice exports: {l >= T_slice} in ascending index order,
    T_slice = the k-th largest slice logit with multiplicity, k = min(top_k,
    V, rows) (1 for greedy)."""
    n = logits_slice.size
    k = 1 if greedy else min(top_k, vocab, n)
    k = max(1, min(k, n))
    T = np.sort(logits_slice)[::-1][k - 1]
    sel = np.nonzero(logits_slice >= T)[0]
    return logits_slice[sel].astype(np.float32), (sel + row0).astype(np.int32)
