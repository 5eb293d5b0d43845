"""CPU restatement of the sequence-parallel regrouping (test infrastructure only).

The reference is single-GPU (it has no collectives anywhere), so this is the oracle for the
build's own token-sharded forward: rank r owns
tokens [r*Lp, (r+1)*Lp) of each batch entry; the B*H (batch, head) units u = b*H + h are
dealt out U = B*H/P per rank (unit u on rank u // U). These functions state the four layout
maps with plain tensor indexing; the CUDA kernels (wdit_ulysses_pack / seq_gather /
seq_scatter / ulysses_unpack) must reproduce them exactly.
"""
from __future__ import annotations

import torch


def units(B: int, H: int, P: int):
    assert (B * H) % P == 0
    U = B * H // P
    return U, [[(u // H, u % H) for u in range(d * U, (d + 1) * U)] for d in range(P)]


def pack(rows: torch.Tensor, B: int, Lp: int, H: int, hd: int, nmat: int, P: int) -> torch.Tensor:
    """rows [B*Lp, >= nmat*H*hd] -> send [P, nmat, U, Lp, hd]."""
    U, owner = units(B, H, P)
    out = torch.empty(P, nmat, U, Lp, hd, dtype=rows.dtype)
    r = rows.view(B, Lp, -1)
    for d in range(P):
        for j, (b, h) in enumerate(owner[d]):
            for c in range(nmat):
                out[d, c, j] = r[b, :, (c * H + h) * hd:(c * H + h + 1) * hd]
    return out


def seq_gather(recv: torch.Tensor, nmat: int, U: int, P: int, Lp: int, hd: int) -> torch.Tensor:
    """recv [P, nmat, U, Lp, hd] -> [nmat, U, P*Lp, hd]."""
    return recv.view(P, nmat, U, Lp, hd).permute(1, 2, 0, 3, 4).reshape(nmat, U, P * Lp, hd)


def seq_scatter(o: torch.Tensor, U: int, P: int, Lp: int, hd: int) -> torch.Tensor:
    """o [U, P*Lp, hd] -> send [P, U, Lp, hd]."""
    return o.view(U, P, Lp, hd).permute(1, 0, 2, 3).contiguous()


def unpack(recv: torch.Tensor, B: int, Lp: int, H: int, hd: int, P: int) -> torch.Tensor:
    """recv [P, U, Lp, hd] (from each unit owner) -> rows [B*Lp, H*hd]."""
    U, owner = units(B, H, P)
    out = torch.empty(B, Lp, H * hd, dtype=recv.dtype)
    rv = recv.view(P, U, Lp, hd)
    for d in range(P):
        for j, (b, h) in enumerate(owner[d]):
            out[b, :, h * hd:(h + 1) * hd] = rv[d, j]
    return out.view(B * Lp, H * hd)
