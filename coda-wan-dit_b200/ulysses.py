"""Token-sharded (sequence-parallel) self-attention with an NCCL Ulysses all-to-all.

Every non-attention op of the Wan block is row-independent, so rank r of P runs the whole
fused GEMM chain on its own tokens [r*Lp, (r+1)*Lp) of each batch entry with no
communication. Self-attention needs all L tokens of a head: the B*H (batch, head) pairs are
dealt out as units (U = B*H/P per rank; Wan-1.3B's 12 heads x CFG batch 2 = 24 units split
evenly over 8 ranks), regrouped with one all-to-all before attention and one after.
Cross-attention needs no exchange (the 512-token context is replicated).

Two transports:

* "p2p" (default): every rank maps its peers' exchange regions once (CUDA IPC) and the
  exchanges are single kernels that store straight into peer memory over NVLink
  (wdit_p2p_qkv_exchange also applies the q/k RMSNorm + RoPE, so the QKV GEMM skips its own
  RMSNorm/RoPE pass), each followed by a bounded stream-ordered wait for all ranks' arrival
  flags (wdit_p2p_wait). With gemm_exchange=True the QKV GEMM itself is the first exchange
  (wdit_gemm_norm_exchange: its epilogue normalizes q / k and stores q, k, v into the owners'
  regions tile by tile). Off by default: on B200 it measures slightly slower than the GEMM
  followed by the exchange kernel (2 GPUs, cfg3: 237.4-237.9 vs 235.9-236.4 ms per forward),
  because the epilogue's peer stores hold back the accumulator release instead of
  overlapping with the tensor-core work.
* "nccl": layout kernels (wdit_ulysses_pack / seq_gather / seq_scatter / ulysses_unpack) move
  the rows into contiguous per-peer blocks and torch.distributed.all_to_all_single (NCCL over
  NVLink / NVSwitch) moves the blocks.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist
import torch.nn.functional as F

from . import _lib, ops
from ._lib import call, ptr, stream_ptr

_HANDLE_BYTES = 64


def _round256(n: int) -> int:
    return (n + 255) // 256 * 256


def exchange_layout(B: int, Lp: int, H: int, hd: int, P: int) -> dict:
    """Byte layout of one rank's exchange region: full[2][3][U][L][hd] bf16, y[2][B*Lp][H*hd]
    bf16, flags[2][P] u32; every part 256-byte aligned (the kernels check it)."""
    U, L, D = B * H // P, P * Lp, H * hd
    full_bytes = 3 * U * L * hd * 2
    y_bytes = B * Lp * D * 2
    fr, yr, fl = _round256(full_bytes), _round256(y_bytes), _round256(4 * P)
    return {
        "full_bytes": full_bytes, "y_bytes": y_bytes,
        "full_off": (0, fr), "y_off": (2 * fr, 2 * fr + yr), "flag_off": (2 * fr + 2 * yr, 2 * fr + 2 * yr + fl),
        "total": 2 * fr + 2 * yr + 2 * fl,
    }


class _Exchange:
    """One rank's exchange region (mapped into every peer) for one (B, Lp, H, hd) shape."""

    def __init__(self, sp: "SeqParallel", B: int, Lp: int, H: int, hd: int, device):
        P, r = sp.world, sp.rank
        self.shape = (B, Lp, H, hd)
        lay = exchange_layout(B, Lp, H, hd, P)
        self.full_bytes, self.y_bytes = lay["full_bytes"], lay["y_bytes"]
        self.full_off, self.y_off, self.flag_off = lay["full_off"], lay["y_off"], lay["flag_off"]
        self.region = torch.empty(lay["total"], dtype=torch.uint8, device=device)
        self.region[self.flag_off[0]:].zero_()
        self.done = torch.zeros(2, dtype=torch.int32, device=device)
        lib = _lib.load()
        handle = ctypes.create_string_buffer(_HANDLE_BYTES)
        off = ctypes.c_longlong(0)
        call("wdit_ipc_handle", ptr(self.region), handle, ctypes.byref(off))
        mine = torch.tensor(list(handle.raw) + list(int(off.value).to_bytes(8, "little")), dtype=torch.uint8,
                            device=device)
        every = torch.empty((P, mine.numel()), dtype=torch.uint8, device=device)
        dist.all_gather_into_tensor(every, mine, group=sp.group)
        every = every.cpu()
        self.opened: list[int] = []
        bases = []
        for p in range(P):
            if p == r:
                bases.append(ptr(self.region))
                continue
            raw = bytes(every[p, :_HANDLE_BYTES].tolist())
            peer_off = int.from_bytes(bytes(every[p, _HANDLE_BYTES:].tolist()), "little")
            base = ctypes.c_void_p(0)
            call("wdit_ipc_open", ctypes.create_string_buffer(raw, _HANDLE_BYTES), ctypes.byref(base))
            self.opened.append(int(base.value))
            bases.append(int(base.value) + peer_off)
        self.peers = (ctypes.c_void_p * P)(*bases)
        self._lib = lib
        torch.cuda.synchronize(device)
        dist.barrier(group=sp.group)  # every region mapped and its flags zeroed before any write

    def flags(self, x: int) -> int:
        return ptr(self.region) + self.flag_off[x]

    def full(self, buf: int, U: int, L: int, hd: int) -> torch.Tensor:
        o = self.full_off[buf]
        return self.region[o:o + self.full_bytes].view(torch.bfloat16).view(3, U, L, hd)

    def y(self, buf: int, rows: int, D: int) -> torch.Tensor:
        o = self.y_off[buf]
        return self.region[o:o + self.y_bytes].view(torch.bfloat16).view(rows, D)

    def close(self) -> None:
        for base in self.opened:
            self._lib.wdit_ipc_close(ctypes.c_void_p(base))
        self.opened = []


class SeqParallel:
    def __init__(self, group, world: int, rank: int, grid: tuple[int, int, int], seq_len: int,
                 transport: str = "p2p", gemm_exchange: bool = False):
        if seq_len % world != 0:
            raise ValueError(f"sequence length {seq_len} is not divisible by {world} ranks")
        if transport not in ("p2p", "nccl"):
            raise ValueError(f"unknown transport {transport!r} (p2p or nccl)")
        self.group = group
        self.world = world
        self.rank = rank
        self.grid = tuple(int(v) for v in grid)
        self.seq_len = seq_len
        self.local_len = seq_len // world
        self.token_offset = rank * self.local_len
        self.transport = transport
        # QKV GEMM storing into the peers' regions itself (p2p transport only)
        self.gemm_exchange = bool(gemm_exchange) and transport == "p2p"
        self._x: _Exchange | None = None
        self.epoch = 0

    def unit_key_mask(self, key_lens, B: int, H: int, L: int, device) -> torch.Tensor | None:
        """Key mask of this rank's (batch, head) units for padded samples: [1, U, 1, L] bool,
        True where key token < the unit's sample length (global lengths, one per batch entry),
        or None when no sample is shorter than L. Unit u = b * H + h lives on rank u // U, so
        this rank's unit j belongs to batch entry (rank * U + j) // H."""
        if key_lens is None:
            return None
        lens = [int(v) for v in key_lens]
        if len(lens) != B:
            raise ValueError(f"{len(lens)} sequence lengths for a batch of {B}")
        if all(n >= L for n in lens):
            return None
        U = B * H // self.world
        unit_len = torch.tensor([lens[(self.rank * U + j) // H] for j in range(U)], device=device)
        return (torch.arange(L, device=device).view(1, 1, 1, L) < unit_len.view(1, U, 1, 1))

    @property
    def fuses_qk_norm(self) -> bool:
        """True when self_attention_p2p takes the raw QKV GEMM output and its RMSNorm partials."""
        return self.transport == "p2p"

    def close(self) -> None:
        """Unmap the peers' exchange regions (call on every rank before destroying the group)."""
        if self._x is not None:
            torch.cuda.synchronize()
            dist.barrier(group=self.group)  # no rank still writes into a region being unmapped
            self._x.close()
            self._x = None

    def self_attention_p2p(self, qkv: torch.Tensor, part: torch.Tensor, wq: torch.Tensor, wk: torch.Tensor,
                           eps: float, cos: torch.Tensor, sin: torch.Tensor, B: int, Lp: int, H: int,
                           hd: int, key_lens=None) -> torch.Tensor:
        """qkv [B*Lp, 3*H*hd] raw QKV GEMM output of this rank's tokens, part [B*Lp, 2*H] its q/k
        mean-square partials -> attention output [B*Lp, H*hd] for the same tokens. key_lens:
        per-sample token counts (keys at or past a sample's count are masked), or None."""
        P = self.world
        assert Lp == self.local_len and (B * H) % P == 0 and hd == 128
        assert qkv.stride(1) == 1 and part.stride(1) == 1 and cos.stride(1) == 1 and sin.stride() == cos.stride()
        # the exchange reads the tables at global token positions up to P * Lp
        assert cos.shape[0] >= P * Lp and sin.shape[0] >= P * Lp, "RoPE tables shorter than the sequence"
        x = self._region(B, Lp, H, hd, qkv.device)
        self.epoch += 1
        e, buf = self.epoch, self.epoch & 1
        st = stream_ptr()
        call("wdit_p2p_qkv_exchange", ptr(qkv), qkv.stride(0), ptr(part), part.stride(0), ptr(wq), ptr(wk),
             float(eps), ptr(cos), ptr(sin), cos.stride(0), B, Lp, H, hd, P, self.rank, x.peers,
             x.full_off[buf], x.flag_off[0], e, ptr(x.done), st)
        return self._attend_and_return(x, buf, e, B, Lp, H, hd, key_lens, qkv.device)

    def self_attention_gemm(self, a: torch.Tensor, w: torch.Tensor, vec: torch.Tensor, ln, wq: torch.Tensor,
                            wk: torch.Tensor, eps: float, cos: torch.Tensor, sin: torch.Tensor, B: int, Lp: int,
                            H: int, hd: int, key_lens=None) -> torch.Tensor:
        """QKV projection + q/k RMSNorm / RoPE + the sequence-to-head exchange in one GEMM launch:
        a [B*Lp, K] this rank's (bf16) tokens, w [3*H*hd, K] the folded QKV weight with its
        per-column vec and LayerNorm fold ln -> attention output [B*Lp, H*hd] for the same
        tokens. key_lens as for self_attention_p2p."""
        P = self.world
        assert self.gemm_exchange and Lp == self.local_len and (B * H) % P == 0 and hd == 128
        assert cos.shape[0] >= P * Lp and sin.shape[0] >= P * Lp, "RoPE tables shorter than the sequence"
        x = self._region(B, Lp, H, hd, a.device)
        self.epoch += 1
        e, buf = self.epoch, self.epoch & 1
        ops.gemm_norm_exchange(a, w, vec=vec, ln=ln, norm_w=(wq, wk), norm_eps=eps, rope_cos=cos, rope_sin=sin,
                               batch=B, Lp=Lp, H=H, P=P, rank=self.rank, peers=x.peers,
                               full_off=x.full_off[buf], flag_off=x.flag_off[0], epoch=e, done_ctr=ptr(x.done))
        return self._attend_and_return(x, buf, e, B, Lp, H, hd, key_lens, a.device)

    def _region(self, B: int, Lp: int, H: int, hd: int, device) -> _Exchange:
        if self._x is None or self._x.shape != (B, Lp, H, hd):
            if self._x is not None:
                self.close()
            self._x = _Exchange(self, B, Lp, H, hd, device)
        return self._x

    def _attend_and_return(self, x: _Exchange, buf: int, e: int, B: int, Lp: int, H: int, hd: int, key_lens,
                           device) -> torch.Tensor:
        """Wait for every rank's q / k / v of epoch e, attend over this rank's units and send the
        outputs back to the ranks owning their tokens."""
        P = self.world
        U, L, D = B * H // P, P * Lp, H * hd
        st = stream_ptr()
        call("wdit_p2p_wait", x.flags(0), P, e, st)
        full = x.full(buf, U, L, hd)
        mask = self.unit_key_mask(key_lens, B, H, L, device)
        o = F.scaled_dot_product_attention(full[0].unsqueeze(0), full[1].unsqueeze(0), full[2].unsqueeze(0),
                                           attn_mask=mask)[0]
        assert o.stride(2) == 1
        call("wdit_p2p_out_exchange", ptr(o), o.stride(0), o.stride(1), B, Lp, H, hd, P, self.rank, x.peers,
             x.y_off[buf], D, x.flag_off[1], e, ptr(x.done) + 4, st)
        call("wdit_p2p_wait", x.flags(1), P, e, st)
        return x.y(buf, B * Lp, D)

    def _a2a(self, out: torch.Tensor, inp: torch.Tensor) -> None:
        if self.world == 1:
            out.copy_(inp)
        else:
            dist.all_to_all_single(out, inp, group=self.group)

    def self_attention(self, qkv: torch.Tensor, B: int, Lp: int, H: int, hd: int, key_lens=None) -> torch.Tensor:
        """qkv [B*Lp, 3*H*hd] (rotated, normalized q/k and v of this rank's tokens) ->
        attention output [B*Lp, H*hd] for the same tokens. key_lens: per-sample token counts
        (keys at or past a sample's count are masked), or None."""
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
        mask = self.unit_key_mask(key_lens, B, H, L, dev)
        o = F.scaled_dot_product_attention(full[0].unsqueeze(0), full[1].unsqueeze(0), full[2].unsqueeze(0),
                                           attn_mask=mask)
        o = o[0]  # [U, L, hd], strides as returned by the attention backend
        assert o.stride(2) == 1
        send2 = torch.empty(P * U * Lp * hd, dtype=torch.bfloat16, device=dev)
        call("wdit_seq_scatter", ptr(o), o.stride(0), o.stride(1), U, P, Lp, hd, ptr(send2), stream_ptr())
        recv2 = torch.empty_like(send2)
        self._a2a(recv2, send2)
        y = torch.empty((B * Lp, D), dtype=torch.bfloat16, device=dev)
        call("wdit_ulysses_unpack", ptr(recv2), B, Lp, H, hd, P, ptr(y), D, stream_ptr())
        return y
