"""Wan2.1 DiT forward on the fused blocks (single GPU or token-sharded over P GPUs).

``FusedWanModel(model)`` takes a model with the stock WanModel attribute layout
(``patch_embedding``, ``text_embedding``, ``time_embedding``, ``time_projection``,
``blocks``, ``head.{head, modulation}``, ``freqs``) and installs ``FusedWanBlock`` for every
block, as the reference does with ``model.blocks = ModuleList([CodaFullBlock(...)])``
(coda_wan/run_wan_coda.py:254-263). ``forward(x_list, t, context_list, seq_len)`` keeps the
stock call signature.

``build_wan(cfg, seed, device)`` creates a randomly initialised model with that layout
(Linear / conv weights ~N(0, 0.02), biases ~N(0, 0.01), modulation ~N(0,1)/sqrt(dim)); there
is no checkpoint here. The non-block parts (patch embedding, text / time embeddings, head,
unpatchify) run as small bf16 / fp32 ops around the blocks; the text MLP and the head use
the fused GEMMs.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops
from .block import Carry, FusedWanBlock
from .ulysses import SeqParallel


@dataclass(frozen=True)
class WanShape:
    dim: int = 1536
    ffn_dim: int = 8960
    num_heads: int = 12
    num_layers: int = 30
    freq_dim: int = 256
    text_dim: int = 4096
    text_len: int = 512
    in_dim: int = 16
    out_dim: int = 16
    patch: tuple = (1, 2, 2)
    eps: float = 1e-6

    @property
    def head_dim(self) -> int:
        return self.dim // self.num_heads


WAN_1_3B = WanShape()
WAN_14B = WanShape(dim=5120, ffn_dim=13824, num_heads=40, num_layers=40)


# ---------------------------------------------------------------------------
# Parameter containers with the stock attribute layout (no forward of their own)
# ---------------------------------------------------------------------------
class _RMSNormParams(nn.Module):
    def __init__(self, dim, eps):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))


class _LayerNormParams(nn.Module):
    def __init__(self, dim, eps, affine):
        super().__init__()
        self.eps = eps
        if affine:
            self.weight = nn.Parameter(torch.ones(dim))
            self.bias = nn.Parameter(torch.zeros(dim))
        else:
            self.register_parameter("weight", None)
            self.register_parameter("bias", None)


class _AttentionParams(nn.Module):
    def __init__(self, dim, num_heads, eps):
        super().__init__()
        self.num_heads = num_heads
        self.eps = eps
        self.window_size = (-1, -1)
        self.q = nn.Linear(dim, dim)
        self.k = nn.Linear(dim, dim)
        self.v = nn.Linear(dim, dim)
        self.o = nn.Linear(dim, dim)
        self.norm_q = _RMSNormParams(dim, eps)
        self.norm_k = _RMSNormParams(dim, eps)


class WanBlockParams(nn.Module):
    def __init__(self, s: WanShape):
        super().__init__()
        self.dim = s.dim
        self.num_heads = s.num_heads
        self.window_size = (-1, -1)
        self.eps = s.eps
        self.norm1 = _LayerNormParams(s.dim, s.eps, False)
        self.self_attn = _AttentionParams(s.dim, s.num_heads, s.eps)
        self.norm3 = _LayerNormParams(s.dim, s.eps, True)
        self.cross_attn = _AttentionParams(s.dim, s.num_heads, s.eps)
        self.norm2 = _LayerNormParams(s.dim, s.eps, False)
        self.ffn = nn.Sequential(nn.Linear(s.dim, s.ffn_dim), nn.GELU(approximate="tanh"), nn.Linear(s.ffn_dim, s.dim))
        self.modulation = nn.Parameter(torch.zeros(1, 6, s.dim))


class _HeadParams(nn.Module):
    def __init__(self, s: WanShape):
        super().__init__()
        self.norm = _LayerNormParams(s.dim, s.eps, False)
        self.head = nn.Linear(s.dim, math.prod(s.patch) * s.out_dim)
        self.modulation = nn.Parameter(torch.zeros(1, 2, s.dim))


def rope_freqs(max_pos: int, head_dim: int, theta: float = 10000.0) -> torch.Tensor:
    """complex128 [max_pos, head_dim/2] rotary frequencies, the head dimension split
    d - 4(d//6), 2(d//6), 2(d//6) = 44/42/42 between frame, height and width."""
    d = head_dim
    cols = []
    for n in (d - 4 * (d // 6), 2 * (d // 6), 2 * (d // 6)):
        expo = torch.arange(0, n, 2, dtype=torch.float64) / n
        ang = torch.outer(torch.arange(max_pos, dtype=torch.float64), torch.pow(theta, -expo))
        cols.append(torch.polar(torch.ones_like(ang), ang))
    return torch.cat(cols, dim=1)


class WanParams(nn.Module):
    def __init__(self, s: WanShape = WAN_1_3B, num_layers: int | None = None):
        super().__init__()
        self.cfg = s
        self.dim = s.dim
        self.num_heads = s.num_heads
        self.patch_embedding = nn.Conv3d(s.in_dim, s.dim, kernel_size=s.patch, stride=s.patch)
        self.text_embedding = nn.Sequential(nn.Linear(s.text_dim, s.dim), nn.GELU(approximate="tanh"),
                                            nn.Linear(s.dim, s.dim))
        self.time_embedding = nn.Sequential(nn.Linear(s.freq_dim, s.dim), nn.SiLU(), nn.Linear(s.dim, s.dim))
        self.time_projection = nn.Sequential(nn.SiLU(), nn.Linear(s.dim, 6 * s.dim))
        n = s.num_layers if num_layers is None else num_layers
        self.blocks = nn.ModuleList([WanBlockParams(s) for _ in range(n)])
        self.head = _HeadParams(s)
        self.register_buffer("freqs", rope_freqs(1024, s.head_dim), persistent=False)


def init_random_(module: nn.Module, seed: int) -> nn.Module:
    """Seeded random init: weights ~N(0, 0.02), biases ~N(0, 0.01), modulation ~N(0,1)/sqrt(dim),
    norm weights 1 and biases 0. Drawn in fp32 on the parameters' device, then cast to each
    parameter's dtype."""
    first = next(module.parameters(), None)
    dev = first.device if first is not None else torch.device("cpu")
    g = torch.Generator(device=dev).manual_seed(seed)
    with torch.no_grad():
        for name, p in module.named_parameters():
            leaf = name.rsplit(".", 1)[-1]
            if "modulation" in name:
                p.copy_(torch.randn(p.shape, generator=g, device=dev) / p.shape[-1] ** 0.5)
            elif "norm" in name:
                p.fill_(1.0 if leaf == "weight" else 0.0)
            elif leaf == "weight":
                p.copy_(0.02 * torch.randn(p.shape, generator=g, device=dev))
            else:
                p.copy_(0.01 * torch.randn(p.shape, generator=g, device=dev))
    return module


def build_wan(s: WanShape = WAN_1_3B, seed: int = 0, device="cuda", num_layers: int | None = None) -> WanParams:
    """Random-init model with the stock layout, bf16 weights (time embedding / projection and
    the modulation vectors fp32, as the stock model keeps them). Built without a CPU copy of
    the weights (the 14B shape is 28 GB in bf16): the parameters are allocated on `device` and
    initialised there."""
    with torch.device("meta"):
        m = WanParams(s, num_layers)
        m.freqs = None  # complex buffer: set on the device below, not cast to bf16
        m = m.to(dtype=torch.bfloat16)
        m.time_embedding.float()
        m.time_projection.float()
        for blk in m.blocks:
            blk.modulation.data = blk.modulation.data.float()
        m.head.modulation.data = m.head.modulation.data.float()
    m = m.to_empty(device=device)
    init_random_(m, seed)
    m.freqs = rope_freqs(1024, s.head_dim).to(device)
    return m


def sinusoidal_embedding(dim: int, pos: torch.Tensor) -> torch.Tensor:
    half = dim // 2
    p = pos.to(torch.float64)
    freq = torch.pow(10000.0, -torch.arange(half, dtype=torch.float64, device=p.device) / half)
    s = torch.outer(p, freq)
    return torch.cat([torch.cos(s), torch.sin(s)], dim=1)


# ---------------------------------------------------------------------------
# Fused model
# ---------------------------------------------------------------------------
class FusedWanModel(nn.Module):
    def __init__(self, model: nn.Module, seq_parallel: SeqParallel | None = None):
        super().__init__()
        self.model = model
        self.carry = Carry()
        self.sp = seq_parallel
        blocks = []
        for b in model.blocks:
            fb = b if isinstance(b, FusedWanBlock) else FusedWanBlock(b, carry=self.carry)
            fb.carry = self.carry
            fb.seq_parallel = seq_parallel
            blocks.append(fb)
        model.blocks = nn.ModuleList(blocks)
        self.dim = int(model.patch_embedding.weight.shape[0])
        self.ckv_all = self._pack_cross_kv(blocks)
        self.patch = tuple(model.patch_embedding.kernel_size)
        # Patch embedding as a GEMM: the Conv3d weight [D, C, pt, ph, pw] flattened to [D, K],
        # K zero-padded to a multiple of 64 (the GEMM's K step); patch_rows builds the A operand.
        pe = model.patch_embedding
        assert tuple(pe.stride) == self.patch, "patch embedding with stride != kernel size"
        wk = pe.weight.detach().reshape(self.dim, -1)
        kp = -(-wk.shape[1] // 64) * 64
        self.w_patch = torch.zeros((self.dim, kp), dtype=torch.bfloat16, device=wk.device)
        self.w_patch[:, :wk.shape[1]] = wk.to(torch.bfloat16)
        self.b_patch = pe.bias.detach().float().contiguous()
        self.out_dim = model.head.head.weight.shape[0] // math.prod(self.patch)
        self.freq_dim = model.time_embedding[0].weight.shape[1]
        te = model.text_embedding
        self.w_t1 = te[0].weight.detach().to(torch.bfloat16)
        self.b_t1 = te[0].bias.detach().float()
        self.w_t2 = te[2].weight.detach().to(torch.bfloat16)
        self.b_t2 = te[2].bias.detach().float()
        self.w_head = model.head.head.weight.detach().to(torch.bfloat16).contiguous()
        self.b_head = model.head.head.bias.detach().float()
        self.head_mod = model.head.modulation.detach().float().reshape(2, self.dim).contiguous()
        self.eps = float(getattr(model.head.norm, "eps", 1e-6))
        # Module.to(dtype) casts a complex buffer to a real dtype (dropping the imaginary part),
        # so keep an own complex128 copy of the rotary frequencies.
        fr = getattr(model, "freqs", None)
        head_dim = self.dim // int(model.num_heads)
        if fr is None or not fr.is_complex():
            fr = rope_freqs(1024, head_dim)
        self.register_buffer("freqs", fr.to(device=model.patch_embedding.weight.device, dtype=torch.complex128),
                             persistent=False)

    # -- embeddings --------------------------------------------------------
    def embed_tokens(self, x_list, seq_len, token_range: tuple[int, int] | None = None):
        """Patch embedding -> [B, rows, dim] bf16 (tokens past a sample's grid are zero), grids,
        true lengths. The Conv3d (kernel = stride = patch) runs as patch rows + one GEMM with the
        bias in its epilogue.

        token_range (lo, hi): embed only tokens [lo, hi) of every sample (a token shard)."""
        lo, hi = token_range if token_range is not None else (0, seq_len)
        rows, B, D = hi - lo, len(x_list), self.dim
        pt, ph, pw = self.patch
        dev = self.w_patch.device
        grids, lens = [], []
        pr = torch.empty((B * rows, self.w_patch.shape[1]), dtype=torch.bfloat16, device=dev)
        for b, u in enumerate(x_list):
            g = (u.shape[1] // pt, u.shape[2] // ph, u.shape[3] // pw)
            grids.append(g)
            lens.append(g[0] * g[1] * g[2])
            ops.patch_rows(u, self.patch, lo, rows, pr.shape[1], out=pr[b * rows:(b + 1) * rows])
        x = torch.empty((B, rows, D), dtype=torch.bfloat16, device=dev)
        valid = [max(0, min(n - lo, rows)) for n in lens]
        if all(v == rows for v in valid):
            ops.gemm_act(pr, self.w_patch, vec=self.b_patch, out=x.view(B * rows, D))
        else:
            for b, v in enumerate(valid):
                if v > 0:
                    ops.gemm_act(pr[b * rows:b * rows + v], self.w_patch, vec=self.b_patch, out=x[b, :v])
                x[b, v:].zero_()
        return x, grids, lens

    def embed_time(self, t: torch.Tensor):
        e = self.model.time_embedding(sinusoidal_embedding(self.freq_dim, t).float())
        e0 = self.model.time_projection(e).unflatten(1, (6, self.dim))
        return e, e0

    def embed_text(self, context_list, text_len):
        ctx = torch.stack([F.pad(u.to(torch.bfloat16), (0, 0, 0, text_len - u.shape[0])) for u in context_list])
        B, Lc, C = ctx.shape
        c = ops.gemm_act(ctx.reshape(B * Lc, C), self.w_t1, vec=self.b_t1, act="gelu_tanh")
        c = ops.gemm_act(c, self.w_t2, vec=self.b_t2, act="none")
        return c.view(B, Lc, self.dim)

    def _pack_cross_kv(self, blocks):
        """Move every block's packed cross-attention K/V weight, bias and K-norm weight into one
        allocation each (the blocks keep views), so one GEMM per forward projects the text
        context for all blocks. None when the blocks do not share shapes and eps."""
        D = self.dim
        if not blocks or any(b.w_ckv.shape != (2 * D, D) or b.rms_eps != blocks[0].rms_eps for b in blocks):
            return None
        L, dev = len(blocks), blocks[0].w_ckv.device
        w_all = torch.empty((L * 2 * D, D), dtype=torch.bfloat16, device=dev)
        b_all = torch.empty(L * 2 * D, dtype=torch.float32, device=dev)
        wk_all = torch.empty((L, D), dtype=torch.float32, device=dev)
        for i, blk in enumerate(blocks):
            rows = slice(i * 2 * D, (i + 1) * 2 * D)
            w_all[rows].copy_(blk.w_ckv)
            b_all[rows].copy_(blk.b_ckv)
            wk_all[i].copy_(blk.w_cnk)
            blk.adopt_cross_kv(w_all[rows], b_all[rows], wk_all[i])
        return w_all, b_all, wk_all, blocks[0].rms_eps

    def cross_kv(self, context: torch.Tensor) -> None:
        """Cross-attention K/V of every block for this forward's text context, in one GEMM and
        one RMSNorm launch; each block takes its columns in its next forward."""
        if self.ckv_all is None:
            return
        w_all, b_all, wk_all, eps = self.ckv_all
        Bc, Lc, D = context.shape
        kv = ops.cross_kv_layers(context.reshape(Bc * Lc, D), w_all, b_all, wk_all, eps)
        for i, blk in enumerate(self.model.blocks):
            blk.set_cross_kv(context, kv[:, i * 2 * D:(i + 1) * 2 * D])

    def _head_fold_specs(self, e, shared_e: bool) -> list[dict]:
        e2 = e.float()
        Be = 1 if shared_e else e2.shape[0]
        return [dict(w=self.w_head, mult_c=1.0, mult_a=self.head_mod[1], mult_b=e2[b], shift_a=self.head_mod[0],
                     shift_b=e2[b], bias=self.b_head) for b in range(Be)]

    def prefold(self, e, e0, shared_e: bool) -> list:
        """All adaLN weight folds of one forward step in one launch: every block's QKV and FFN1
        folds (handed to the blocks for their next forward with this e0) and the head's fold
        (returned). They depend only on the step's time embedding."""
        specs, owners = [], []
        for blk in self.model.blocks:
            sp = blk.fold_specs(e0)
            owners.append((blk, len(specs), len(sp)))
            specs += sp
        head_first = len(specs)
        specs += self._head_fold_specs(e, shared_e)
        folds = ops.fold_weight_batch(specs)
        for blk, i0, n in owners:
            blk.set_prefolded(e0, folds[i0:i0 + n])
        return folds[head_first:]

    def head(self, x32, e, carry_stats, rows, shared_e: bool, folds: list | None = None):
        """LayerNorm + 2-vector modulation + Linear(dim -> prod(patch)*out_dim), LN absorbed.
        `folds`: this head's weight folds from `prefold` (computed here when absent)."""
        xb, stats = carry_stats
        specs = self._head_fold_specs(e, shared_e)
        Be = len(specs)
        outs = []
        per = rows // Be
        for b in range(Be):
            r0, r1 = b * per, (b + 1) * per
            if folds is not None and len(folds) == Be:
                wf, cs, vec = folds[b]
            else:
                sp = specs[b]
                wf, cs, vec = ops.fold_weight(sp["w"], mult_c=1.0, mult_a=sp["mult_a"], mult_b=sp["mult_b"],
                                              shift_a=sp["shift_a"], shift_b=sp["shift_b"], bias=sp["bias"])
            outs.append(ops.gemm_act(xb[r0:r1], wf, vec=vec, act="none", ln=ops.LnFold(cs, stats[r0:r1], self.eps)))
        return torch.cat(outs) if len(outs) > 1 else outs[0]

    def unpatchify(self, y, grids, lens, rows_per_batch):
        pt, ph, pw = self.patch
        c = self.out_dim
        outs = []
        for i, ((f, h, w), n) in enumerate(zip(grids, lens)):
            u = y[i * rows_per_batch: i * rows_per_batch + n].view(f, h, w, pt, ph, pw, c)
            u = torch.einsum("fhwpqrc->cfphqwr", u)
            outs.append(u.reshape(c, f * pt, h * ph, w * pw))
        return outs

    # -- forward -----------------------------------------------------------
    def forward(self, x_list, t, context_list, seq_len, text_len: int = 512, return_tokens: bool = False):
        """Stock signature. With token sharding (or return_tokens=True) the result is the head's
        per-token output [B, L(local), prod(patch) * out_dim] instead of unpatchified latents."""
        dev = self.model.patch_embedding.weight.device
        B = len(x_list)
        t = torch.as_tensor(t).reshape(-1)
        # CFG: entries that share the timestep share the modulation (one weight fold per block).
        # The check reads host values (one sync if t lives on the device).
        tv = t.tolist()
        shared_e = all(v == tv[0] for v in tv)
        t = t.to(dev)
        sp = self.sp
        token_range = None if sp is None else (sp.token_offset, sp.token_offset + sp.local_len)
        x, grids, lens = self.embed_tokens(x_list, seq_len, token_range)
        if sp is not None and any(tuple(g) != tuple(sp.grid) for g in grids):
            raise ValueError(f"token sharding was set up for grid {tuple(sp.grid)}; the samples have grids {grids}")
        e, e0 = self.embed_time(t[:1] if shared_e else t)
        head_folds = self.prefold(e, e0, shared_e)
        context = self.embed_text(context_list, text_len)
        self.cross_kv(context)
        Lx = x.shape[1]
        # Per-sample token counts (global, also under token sharding, where the gathered-head
        # attention masks each unit's keys past its sample's count); None when no sample is padded.
        grid_sizes = torch.tensor(grids, dtype=torch.long)
        seq_lens_arg = torch.tensor(lens, dtype=torch.long) if any(n != seq_len for n in lens) else None
        x = x.contiguous()
        for blk in self.model.blocks:
            x = blk(x, e0, seq_lens_arg, grid_sizes, self.freqs, context, None)
        x32 = x.reshape(B * Lx, self.dim)
        carried = self.carry.get(x32)
        y = self.head(x32, e, carried, B * Lx, shared_e, head_folds)
        if sp is not None or return_tokens:
            return y.view(B, Lx, -1)
        return [u.float() for u in self.unpatchify(y, grids, lens, Lx)]
