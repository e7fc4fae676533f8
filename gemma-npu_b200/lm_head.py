"""Column-sharded LM head across GPUs: local int8 GEMV + NCCL all-gather of the logits.

The reference computes the whole 262144-wide LM head on one CPU
(Int8Head, gemma_npu.py:159-172; softcap pipeline.py:335-338).  Here rank g of a
G-rank process group holds rows [g*V/G, (g+1)*V/G) of the [V, K] head weight
(V/G a whole number of rows, padded up when V % G != 0), computes its slice of
the softcapped fp32 logits with the fused GEMV, and an all-gather over
NVLink/NVSwitch assembles the full [V] vector on every rank.  One process per
GPU; the process group is torch.distributed's (NCCL on GPUs).

Two transports for the all-gather:
  "nccl"  the GEMV into a local slice, then torch.distributed.all_gather_into_tensor;
  "peer"  one kernel (w8_lm_head_peer_f32): the GEMV stores every logit straight into
          every rank's gathered buffer through CUDA IPC peer pointers (plain stores over
          NVLink), with ready / done flags in the same buffers; the greedy token comes out
          of the same kernel.  The process group is used only once, to exchange the
          buffers' IPC handles.
"""
import ctypes

import torch
import torch.distributed as dist

from . import _lib, kernels
from .gemm import quantize_weight

TRANSPORTS = ("nccl", "peer")


def shard_rows(vocab, world, rank):
    """Row range [r0, r1) of the head weight owned by `rank`; shards are ceil(V/G) rows
    rounded up to a multiple of 4 (so every shard starts on a 16-byte boundary of the
    gathered fp32 logits), the last one shorter."""
    per = -(-vocab // world)
    per = -(-per // 4) * 4
    r0 = min(rank * per, vocab)
    return r0, min(r0 + per, vocab), per


def gather_logits(local, full, vocab, group=None):
    """All-gather equal-length per-rank logit slices into `full` and return its first `vocab`.

    `local` is this rank's [per] slice (a short last shard zero-padded), `full` a
    [world * per] buffer on the same device; rank order is shard order.
    """
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return local[:vocab]
    dist.all_gather_into_tensor(full, local, group=group)
    return full[:vocab]


class _Device1D:
    """A raw device allocation seen as a 1-D torch tensor (no copy), via the CUDA array
    interface; the allocation stays owned by whoever made it."""

    def __init__(self, ptr, n, typestr):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (ptr, False), "version": 3}


class PeerBuffers:
    """Every rank's gathered-logits buffer of w8_lm_head_peer_f32: this rank's own
    (w8_peer_alloc) and the others mapped from their IPC handles (w8_peer_open), in rank
    order.  `logits` is this rank's [vocab] fp32 view.  close() unmaps and frees; every
    rank calls it (it synchronises the group)."""

    def __init__(self, vocab, group=None, device=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = device
        nbytes = _lib.lib().w8_lm_head_peer_bytes(vocab)
        own = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(64)
        _lib.check(_lib.lib().w8_peer_alloc(nbytes, ctypes.byref(own), handle), "w8_peer_alloc")
        self.own = own.value
        handles = [None] * self.world
        dist.all_gather_object(handles, handle.raw, group=group)
        self.ptrs, self.opened = [], []
        for r, h in enumerate(handles):
            if r == self.rank:
                self.ptrs.append(self.own)
                continue
            p = ctypes.c_void_p()
            _lib.check(_lib.lib().w8_peer_open(ctypes.create_string_buffer(h, 64), ctypes.byref(p)), "w8_peer_open")
            self.ptrs.append(p.value)
            self.opened.append(p.value)
        self.table = (ctypes.c_void_p * self.world)(*self.ptrs)
        self.logits = torch.as_tensor(_Device1D(self.own, vocab, "<f4"), device=device)
        dist.barrier(group=group)

    def close(self):
        if self.own is None:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)  # no rank writes into a buffer any more
        for p in self.opened:
            _lib.check(_lib.lib().w8_peer_close(p), "w8_peer_close")
        dist.barrier(group=self.group)  # every mapping of this rank's buffer is gone
        self.logits = None
        _lib.check(_lib.lib().w8_peer_free(self.own), "w8_peer_free")
        self.own, self.opened = None, []


class ShardedInt8Head:
    """The int8 LM head split by output rows over the ranks of a process group.

    transport "nccl" gathers the logits with NCCL after the GEMV; "peer" stores them into
    every rank's buffer from inside the GEMV (one kernel, see the module docstring).  With
    "peer", every rank makes the same calls in the same order, and the logits a call
    returns are valid until this rank's next call.
    """

    def __init__(self, weight, group=None, device=None, cap=0.0, transport="nccl"):
        if transport not in TRANSPORTS:
            raise ValueError(f"transport must be one of {TRANSPORTS}")
        self.transport = transport
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.vocab, self.hidden = weight.shape
        self.r0, self.r1, self.per = shard_rows(self.vocab, self.world, self.rank)
        self.cap = float(cap or 0.0)
        self.device = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        self.wq, sw = quantize_weight(weight[self.r0: self.r1], self.device)
        self.sw = sw.to(torch.bfloat16)
        # Gather target: world x per slots (the last shard may be short: its tail is zero).
        self.full = torch.empty(self.world * self.per, dtype=torch.float32, device=self.device)
        self.local = torch.zeros(self.per, dtype=torch.float32, device=self.device)
        self.peer = None
        if transport == "peer" and self.world > 1:
            self.peer = PeerBuffers(self.vocab, group, self.device)
            self.best = torch.zeros((1,), dtype=torch.int64, device=self.device)

    def _peer_call(self, h, best, keys_only=False):
        h = h.reshape(-1).to(torch.bfloat16).contiguous()
        n = self.r1 - self.r0
        entry = "w8_lm_head_peer_argmax" if keys_only else "w8_lm_head_peer_f32"
        _lib.call(entry, h.data_ptr(), self.wq.data_ptr() if n else None, self.sw.data_ptr(),
                  self.cap, n, self.hidden, self.r0, self.vocab, self.world, self.rank, self.peer.table,
                  best.data_ptr() if best is not None else None, torch.cuda.current_stream(self.device).cuda_stream)
        return self.peer.logits

    def close(self):
        """Release the peer buffers (transport "peer"); every rank calls it."""
        if self.peer is not None:
            self.peer.close()
            self.peer = None

    def local_logits(self, h):
        """This rank's softcapped fp32 logits [r1 - r0] of one hidden row."""
        n = self.r1 - self.r0
        if n > 0:
            kernels.lm_head_logits(h, self.wq, self.sw, self.cap, out=self.local[:n])
        return self.local

    def __call__(self, h):
        """Full fp32 logits [V] of one hidden row on every rank."""
        if self.peer is not None:
            return self._peer_call(h, None)
        return gather_logits(self.local_logits(h), self.full, self.vocab, self.group)

    def greedy(self, h):
        """The greedy token (gemma_npu.py:291, logits.argmax()) without gathering the logits:
        each rank folds its shard's argmax inside the head GEMV, re-keys it with the global
        row id, and one 8-byte all-gather per rank picks the winner (ties: lowest id).
        With transport "peer" only the keys travel, inside the head kernel
        (w8_lm_head_peer_argmax); the logits stay on their rank."""
        if self.peer is not None:
            self._peer_call(h, self.best, keys_only=True)
            return (0xFFFFFFFF - (self.best.reshape(()) & 0xFFFFFFFF))
        n = self.r1 - self.r0
        if n > 0:
            _, best = kernels.lm_head_logits(h, self.wq, self.sw, self.cap, out=self.local[:n], argmax="key")
            key = shard_key(best, self.r0)
        else:
            key = torch.full((1,), -(1 << 63), dtype=torch.int64, device=self.device)
        return greedy_from_keys(key, self.group)


def shard_key(best, r0):
    """A shard's packed key (unsigned: monotone value bits << 32 | 2^32 - 1 - local row) as a
    signed-comparable int64 with the global row id r0 + local row."""
    return (best - r0) ^ (-(1 << 63))


def merge_key(high, token):
    """Signed-comparable packed key of (monotone value bits, global token id): larger is
    better, ties to the lower id."""
    return (((high.to(torch.int64) & 0xFFFFFFFF) << 32) | (0xFFFFFFFF - token.to(torch.int64))) ^ (-(1 << 63))


def greedy_from_keys(key, group=None):
    """Winner among the ranks' packed keys: the token id of the largest key."""
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        keys = torch.empty((dist.get_world_size(group),), dtype=torch.int64, device=key.device)
        dist.all_gather_into_tensor(keys, key.reshape(1), group=group)
        key = keys.max()
    return (0xFFFFFFFF - (key.reshape(()) & 0xFFFFFFFF))
