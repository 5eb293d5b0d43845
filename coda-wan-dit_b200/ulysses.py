"""Token-sharded (sequence-parallel) self-attention with an NCCL Ulysses all-to-all.

Every non-attention op of the Wan block is row-independent, so rank r of P runs the whole
fused GEMM chain on its own tokens [r*Lp, (r+1)*Lp) of each batch entry with no
communication. Self-attention needs all L tokens of a head: the B*H (batch, head) pairs are
dealt out as units (U = B*H/P per rank; Wan-1.3B's 12 heads x CFG batch 2 = 24 units split
evenly over 8 ranks), regrouped with one all-to-all before attention and one after.
Cross-attention needs no exchange (the 512-token context is replicated).

Layout kernels (wdit_ulysses_pack / seq_gather / seq_scatter / ulysses_unpack) move the
rows into contiguous per-peer blocks; torch.distributed.all_to_all_single (NCCL over
NVLink / NVSwitch) moves the blocks.
"""
from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn.functional as F

from ._lib import call, ptr, stream_ptr


class SeqParallel:
    def __init__(self, group, world: int, rank: int, grid: tuple[int, int, int], seq_len: int):
        if seq_len % world != 0:
            raise ValueError(f"sequence length {seq_len} is not divisible by {world} ranks")
        self.group = group
        self.world = world
        self.rank = rank
        self.grid = tuple(int(v) for v in grid)
        self.seq_len = seq_len
        self.local_len = seq_len // world
        self.token_offset = rank * self.local_len

    def _a2a(self, out: torch.Tensor, inp: torch.Tensor) -> None:
        if self.world == 1:
            out.copy_(inp)
        else:
            dist.all_to_all_single(out, inp, group=self.group)

    def self_attention(self, qkv: torch.Tensor, B: int, Lp: int, H: int, hd: int) -> torch.Tensor:
        """qkv [B*Lp, 3*H*hd] (rotated, normalized q/k and v of this rank's tokens) ->
        attention output [B*Lp, H*hd] for the same tokens."""
        P = self.world
        assert Lp == self.local_len and (B * H) % P == 0
        U = B * H // P
        D = H * hd
        L = P * Lp
        dev = qkv.device
        send = torch.empty(P * 3 * U * Lp * hd, dtype=torch.bfloat16, device=dev)
        call("wdit_ulysses_pack", ptr(qkv), qkv.stride(0), B, Lp, H, hd, 3, P, ptr(send), stream_ptr())
        recv = torch.empty_like(send)
        self._a2a(recv, send)
        full = torch.empty((3, U, L, hd), dtype=torch.bfloat16, device=dev)
        call("wdit_seq_gather", ptr(recv), 3, U, P, Lp, hd, ptr(full), stream_ptr())
        o = F.scaled_dot_product_attention(full[0].unsqueeze(0), full[1].unsqueeze(0), full[2].unsqueeze(0))
        o = o[0]  # [U, L, hd], strides as returned by the attention backend
        assert o.stride(2) == 1
        send2 = torch.empty(P * U * Lp * hd, dtype=torch.bfloat16, device=dev)
        call("wdit_seq_scatter", ptr(o), o.stride(0), o.stride(1), U, P, Lp, hd, ptr(send2), stream_ptr())
        recv2 = torch.empty_like(send2)
        self._a2a(recv2, send2)
        y = torch.empty((B * Lp, D), dtype=torch.bfloat16, device=dev)
        call("wdit_ulysses_unpack", ptr(recv2), B, Lp, H, hd, P, ptr(y), D, stream_ptr())
        return y
