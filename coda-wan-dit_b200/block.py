"""Drop-in fused Wan2.1 attention block for B200.

``FusedWanBlock(inner, rope_cos=None, rope_sin=None)`` wraps a stock ``WanAttentionBlock``
(anything with its attribute layout: ``self_attn.{q,k,v,o,norm_q,norm_k}``,
``cross_attn.{...}``, ``norm3``, ``ffn[0]``, ``ffn[2]``, ``modulation``, ``eps``,
``num_heads``) and keeps its forward signature
``forward(x, e, seq_lens, grid_sizes, freqs, context, context_lens) -> x``.
Counterpart of coda_wan/run_wan_coda.py:82-205 (CodaFullBlock).

Per block, on one stream (M = B * L rows):

    fold QKV weight      W' = W * (1 + mod1 + e1), csum, vec = (mod0 + e0)^T W + b (inside a
                         model the folds of all blocks run in one launch per step instead)
    QKV GEMM             LN absorbed + bias -> qkv bf16 + q/k mean-square partials, then the
                         in-place full-width q/k RMSNorm + 3D RoPE pass
    self-attention       PyTorch SDPA (or the Ulysses all-to-all around it)
    self-O GEMM          x += (y Wo^T + bo) * (mod2 + e2)   -> x fp32, bf16 copy, LN stats
    cross-Q GEMM         norm3 folded statically (gamma into W, beta into vec) + RMSNorm
    cross-KV GEMM        context -> k (RMSNorm), v (inside a model: one GEMM for all blocks)
    cross-attention      PyTorch SDPA
    cross-O GEMM         x += cy Wco^T + bco                 -> x, bf16 copy, LN stats
    fold FFN1 weight     as QKV with (mod4 + e4, mod3 + e3)
    FFN1 GEMM            LN absorbed + shift term, tanh-GELU  -> h bf16
    FFN2 GEMM            x += (h W2^T + b2) * (mod5 + e5)    -> x, bf16 copy, LN stats

The LayerNorm statistics and the bf16 copy of the residual stream produced by each residual
epilogue are handed to the next block through a ``Carry`` keyed on the residual tensor object
(weakly referenced) and its version counter, so only the first block runs the standalone
statistics pass.

Differences from the reference's block, all deliberate:
  * batch > 1 (CFG) and any grid are accepted; ``freqs`` is used (the reference asserts
    batch 1 and a fixed grid, and drops freqs, coda_wan/run_wan_coda.py:140-141);
  * grid sizes / sequence lengths are read once per distinct tensor (not one device sync
    per block);
  * like the reference (:169), an fp32 input ``x`` is updated in place.
"""
from __future__ import annotations

import threading
import weakref

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops

_ONE_SYNC = threading.local()


def _root(t: torch.Tensor) -> torch.Tensor:
    """The tensor object that owns the storage of `t` (views point to it through ``_base``)."""
    return t._base if t._base is not None else t


def _host_values(t):
    """Python ints of a small tensor, read once per distinct tensor object and version.

    The cache entry holds a weak reference to the tensor it was read from: a new tensor that
    happens to get the same ``id`` and address after the old one was freed is a miss."""
    if t is None:
        return None
    if not torch.is_tensor(t):
        return [list(v) if isinstance(v, (list, tuple)) else int(v) for v in t]
    cache = getattr(_ONE_SYNC, "cache", None)
    if cache is None:
        cache = _ONE_SYNC.cache = {}
    hit = cache.get(id(t))
    if hit is not None and hit[0]() is t and hit[1] == t._version:
        return hit[2]
    if len(cache) > 64:
        cache.clear()
    vals = t.tolist()
    cache[id(t)] = (weakref.ref(t), t._version, vals)
    return vals


class Carry:
    """bf16 copy + LayerNorm statistics of the residual stream, valid for one tensor state.

    The key is the residual tensor itself (a weak reference to the tensor object that owns
    its storage, so any view of it matches) and its version counter. The residual epilogues
    update the fp32 stream in place through the C ABI, which torch does not see, so the block
    bumps the version itself after its last write (``torch.autograd.graph.increment_version``)
    and records the bumped version. A freed tensor whose address is reused by a new tensor,
    or a tensor changed in place by torch ops since, is a miss: its statistics are recomputed.
    """

    def __init__(self):
        self.ref = None
        self.version = -1
        self.shape = None
        self.xb = None
        self.stats = None

    def get(self, x: torch.Tensor):
        if self.ref is None or x.dtype != torch.float32:
            return None
        if self.ref() is _root(x) and self.version == x._version and self.shape == tuple(x.shape):
            return self.xb, self.stats
        return None

    def put(self, x: torch.Tensor, xb: torch.Tensor, stats: torch.Tensor) -> None:
        self.ref = weakref.ref(_root(x))
        self.version = x._version
        self.shape = tuple(x.shape)
        self.xb = xb
        self.stats = stats


_DEFAULT_CARRY = threading.local()


def default_carry() -> Carry:
    """Per-thread carry shared by standalone blocks (blocks installed one by one, as the
    reference installs its CodaFullBlock, hand the statistics of their output to the next
    block through it)."""
    c = getattr(_DEFAULT_CARRY, "carry", None)
    if c is None:
        c = _DEFAULT_CARRY.carry = Carry()
    return c


def local_attention(q, k, v, k_lens=None):
    """q [B, Lq, H, hd] (any strides, last dim contiguous) -> [B, Lq, H, hd] via PyTorch SDPA."""
    mask = None
    B, Lk = k.shape[0], k.shape[1]
    if k_lens is not None:
        lens = _host_values(k_lens)
        if any(int(l) < Lk for l in lens):
            kl = torch.tensor([int(l) for l in lens], device=q.device).view(B, 1, 1, 1)
            mask = torch.arange(Lk, device=q.device).view(1, 1, 1, Lk) < kl
    o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), attn_mask=mask)
    return o.transpose(1, 2)


def _bf16_param(p: torch.Tensor) -> torch.Tensor:
    return p.detach() if p.dtype == torch.bfloat16 else p.detach().to(torch.bfloat16)


class FusedWanBlock(nn.Module):
    def __init__(self, inner: nn.Module, rope_cos: torch.Tensor | None = None, rope_sin: torch.Tensor | None = None,
                 carry: Carry | None = None):
        super().__init__()
        self.inner = inner
        sa, ca = inner.self_attn, inner.cross_attn
        dev = sa.q.weight.device
        if dev.type != "cuda":
            raise RuntimeError("FusedWanBlock needs the wrapped block on a CUDA device")
        self.dim = int(sa.q.weight.shape[0])
        self.num_heads = int(inner.num_heads)
        self.head_dim = self.dim // self.num_heads
        self.ffn_dim = int(inner.ffn[0].weight.shape[0])
        self.eps = float(inner.eps)
        self.rms_eps = float(getattr(sa, "eps", inner.eps))
        self.carry = carry  # None: the per-thread default carry
        self.workspace = None  # None: the per-device shared workspace (launches are stream-ordered)
        self.seq_parallel = None  # set by the model for token-sharded runs
        self.kernel_timer = None  # list: (start event, end event, flops) of each FFN1 GEMM launch
        # (e, folds) set by the model for the next forward: this step's QKV / FFN1 weight folds,
        # computed for all blocks in one launch (`fold_specs`); used when forward gets that e.
        self._prefolded = None
        # (context, kv) set by the model: this block's cross-attention K (normalized) and V,
        # projected for all blocks in one GEMM; used when forward gets that context.
        self._pre_ckv = None

        # Zero-copy where the weights are already bf16: QKV and cross-KV are packed into
        # one allocation each and the Linear parameters become views of it.
        if sa.q.weight.dtype == torch.bfloat16:
            wqkv, bqkv = ops.prepack_qkv_inplace(sa.q, sa.k, sa.v)
        else:
            wqkv = torch.cat([_bf16_param(sa.q.weight), _bf16_param(sa.k.weight), _bf16_param(sa.v.weight)])
            bqkv = torch.cat([sa.q.bias.detach(), sa.k.bias.detach(), sa.v.bias.detach()])
        self.register_buffer("w_qkv", wqkv, persistent=False)
        self.register_buffer("b_qkv", bqkv.float().contiguous(), persistent=False)
        self.register_buffer("w_o", _bf16_param(sa.o.weight), persistent=False)
        self.register_buffer("b_o", sa.o.bias.detach().float().contiguous(), persistent=False)
        self.register_buffer("w_nq", sa.norm_q.weight.detach().float().contiguous(), persistent=False)
        self.register_buffer("w_nk", sa.norm_k.weight.detach().float().contiguous(), persistent=False)

        if ca.k.weight.dtype == torch.bfloat16:
            wkv = torch.cat([ca.k.weight.detach(), ca.v.weight.detach()]).contiguous()
            bkv = torch.cat([ca.k.bias.detach(), ca.v.bias.detach()]).contiguous()
            d = self.dim
            ops.replace_parameter_with_view(ca.k, "weight", wkv[:d])
            ops.replace_parameter_with_view(ca.v, "weight", wkv[d:])
            ops.replace_parameter_with_view(ca.k, "bias", bkv[:d])
            ops.replace_parameter_with_view(ca.v, "bias", bkv[d:])
        else:
            wkv = torch.cat([_bf16_param(ca.k.weight), _bf16_param(ca.v.weight)])
            bkv = torch.cat([ca.k.bias.detach(), ca.v.bias.detach()])
        self.register_buffer("w_ckv", wkv, persistent=False)
        self.register_buffer("b_ckv", bkv.float().contiguous(), persistent=False)
        self.register_buffer("w_cnq", ca.norm_q.weight.detach().float().contiguous(), persistent=False)
        self.register_buffer("w_cnk", ca.norm_k.weight.detach().float().contiguous(), persistent=False)
        self.register_buffer("w_co", _bf16_param(ca.o.weight), persistent=False)
        self.register_buffer("b_co", ca.o.bias.detach().float().contiguous(), persistent=False)

        # norm3 (affine LayerNorm) folded once: W' = W diag(gamma), vec = beta^T W + b.
        n3 = inner.norm3
        w_cq = _bf16_param(ca.q.weight)
        self.cross_ln = not isinstance(n3, nn.Identity)
        if self.cross_ln:
            gamma = n3.weight.detach().float().contiguous() if getattr(n3, "weight", None) is not None else \
                torch.ones(self.dim, device=dev)
            beta = n3.bias.detach().float().contiguous() if getattr(n3, "bias", None) is not None else \
                torch.zeros(self.dim, device=dev)
            self.cross_eps = float(getattr(n3, "eps", self.eps))
            wf, cs, vec = ops.fold_weight(w_cq.contiguous(), mult_c=0.0, mult_a=gamma, shift_a=beta,
                                          bias=ca.q.bias.detach().float())
            self.register_buffer("w_cq", wf, persistent=False)
            self.register_buffer("csum_cq", cs, persistent=False)
            self.register_buffer("vec_cq", vec, persistent=False)
        else:
            self.register_buffer("w_cq", w_cq, persistent=False)
            self.register_buffer("vec_cq", ca.q.bias.detach().float().contiguous(), persistent=False)

        self.register_buffer("w_1", _bf16_param(inner.ffn[0].weight), persistent=False)
        self.register_buffer("b_1", inner.ffn[0].bias.detach().float().contiguous(), persistent=False)
        self.register_buffer("w_2", _bf16_param(inner.ffn[2].weight), persistent=False)
        self.register_buffer("b_2", inner.ffn[2].bias.detach().float().contiguous(), persistent=False)
        self.register_buffer("mod", inner.modulation.detach().float().reshape(6, self.dim).contiguous(),
                             persistent=False)
        self._rope = {}
        if rope_cos is not None and rope_sin is not None:
            # the reference's token-major [tokens, 64] tables are the kernel's layout
            self._rope["given"] = (rope_cos.float().contiguous(), rope_sin.float().contiguous())

    # ------------------------------------------------------------------
    def _carry(self) -> Carry:
        return self.carry if self.carry is not None else default_carry()

    def _rope_tables(self, grid, freqs, rows: int):
        """Token-major cos / sin tables of `grid` with at least `rows` rows: tokens past the grid
        (padding up to the sequence length) get the identity rotation (cos 1, sin 0)."""
        if "given" in self._rope:
            return self._rope["given"]
        key = (tuple(grid), freqs.data_ptr(), rows)
        tab = self._rope.get(key)
        if tab is None:
            cos, sin = ops.build_wan_rope_table(grid, freqs)
            if cos.shape[0] < rows:
                pad = rows - cos.shape[0]
                cos = torch.cat([cos, cos.new_ones((pad, cos.shape[1]))])
                sin = torch.cat([sin, sin.new_zeros((pad, sin.shape[1]))])
            tab = (cos, sin)
            if len(self._rope) > 8:
                self._rope = {}
            self._rope[key] = tab
        return tab

    def _input_stats(self, x2: torch.Tensor):
        """bf16 copy, fp32 residual buffer and LN statistics of the block input rows."""
        M, D = x2.shape
        hit = self._carry().get(x2)
        if hit is not None:
            xb, stats = hit
            return x2, xb, stats
        stats = torch.empty((M, ops.stats_tiles(D), 2), dtype=torch.float32, device=x2.device)
        if x2.dtype == torch.float32:
            x32 = x2 if x2.is_contiguous() else x2.contiguous()
            xb = torch.empty((M, D), dtype=torch.bfloat16, device=x2.device)
            ops.ln_stats(x32, stats_out=stats, x_bf16_out=xb)
        else:
            xb = x2.to(torch.bfloat16).contiguous()
            x32 = torch.empty((M, D), dtype=torch.float32, device=x2.device)
            ops.ln_stats(xb, stats_out=stats, x_f32_out=x32)
        return x32, xb, stats

    def fold_specs(self, e: torch.Tensor) -> list[dict]:
        """The per-step adaLN weight folds of this block for modulation e [Be, 6, D]
        (`ops.fold_weight_batch` specs): QKV then FFN1 for each of the Be entries."""
        D = self.dim
        ev = e.float().reshape(-1, 6 * D).contiguous()
        mod = self.mod
        specs = []
        for b in range(ev.shape[0]):
            specs.append(dict(w=self.w_qkv, mult_c=1.0, mult_a=mod[1], mult_b=ev[b, D:2 * D], shift_a=mod[0],
                              shift_b=ev[b, :D], bias=self.b_qkv))
            specs.append(dict(w=self.w_1, mult_c=1.0, mult_a=mod[4], mult_b=ev[b, 4 * D:5 * D], shift_a=mod[3],
                              shift_b=ev[b, 3 * D:4 * D], bias=self.b_1))
        return specs

    def adopt_cross_kv(self, w: torch.Tensor, b: torch.Tensor, wk: torch.Tensor) -> None:
        """Move the packed cross-attention K/V weight, its fp32 bias and the K norm weight into
        the given storage (the model's all-blocks allocations; same values). The wrapped module's
        bf16 K/V weights, views of the old packed weight, become views of the new one."""
        ca, d = self.inner.cross_attn, self.dim
        if ca.k.weight.dtype == torch.bfloat16 and ca.k.weight.untyped_storage().data_ptr() == \
                self.w_ckv.untyped_storage().data_ptr():
            ops.replace_parameter_with_view(ca.k, "weight", w[:d])
            ops.replace_parameter_with_view(ca.v, "weight", w[d:])
        self.w_ckv, self.b_ckv, self.w_cnk = w, b, wk

    def set_cross_kv(self, context: torch.Tensor, kv: torch.Tensor) -> None:
        """Hand this block its cross-attention K/V of `context` for its next forward."""
        self._pre_ckv = (context, kv)

    def set_prefolded(self, e: torch.Tensor, folds: list) -> None:
        """Hand this block the results of its `fold_specs(e)` for its next forward."""
        self._prefolded = (e, folds)

    def forward(self, x, e, seq_lens, grid_sizes, freqs, context, context_lens):
        B, L, D = x.shape
        H, hd = self.num_heads, self.head_dim
        M = B * L
        dev = x.device
        sp = self.seq_parallel
        x32, xb, stats = self._input_stats(x.reshape(M, D))

        # Modulation rows: e [Be, 6, D] fp32 with Be in {1, B}.
        ev = e.float().reshape(-1, 6 * D)
        Be = ev.shape[0]
        assert Be in (1, B), "e must have batch 1 (shared modulation) or the block's batch"
        ev = ev.contiguous()
        mod = self.mod
        pre, self._prefolded = self._prefolded, None
        folds = pre[1] if pre is not None and pre[0] is e and len(pre[1]) == 2 * Be else None
        gate_stride = 6 * D
        rows_per_batch = L if Be == B and B > 1 else M

        def e_row(b, i):
            return ev[b, i * D:(i + 1) * D]

        # --- rope table rows for this (possibly token-sharded) block ---
        # One table for all samples when they share a grid; otherwise each sample's rows are
        # projected with its own grid's table (stock Wan applies each sample's own grid).
        if sp is not None:
            grid, token_offset, grid_rows_per_batch = sp.grid, sp.token_offset, L
            sample_grids = None
            cos, sin = self._rope_tables(grid, freqs, sp.seq_len)
        else:
            grids = [tuple(int(v) for v in g) for g in _host_values(grid_sizes)]
            token_offset, grid_rows_per_batch = 0, L
            sample_grids = grids if len(set(grids)) > 1 else None
            if sample_grids is not None and len(sample_grids) != B:
                raise ValueError(f"{len(sample_grids)} grid sizes for a batch of {B}")
            cos, sin = self._rope_tables(grids[0], freqs, L)

        # --- self-attention branch ---
        # QKV row segments: one per modulation row (Be) or, with per-sample grids, one per sample
        nseg = B if sample_grids is not None else Be
        # With the NVLink peer-store exchange the q/k RMSNorm + RoPE happen inside the exchange:
        # either the QKV GEMM stores into the owners' regions itself (one segment), or the GEMM
        # only emits the raw projection and its mean-square partials for the exchange kernel.
        fused_exchange = sp is not None and sp.fuses_qk_norm
        if fused_exchange and sp.gemm_exchange and nseg == 1 and D % 256 == 0:
            wf, cs, vec = folds[0] if folds is not None else ops.fold_weight(
                self.w_qkv, mult_c=1.0, mult_a=mod[1], mult_b=e_row(0, 1), shift_a=mod[0], shift_b=e_row(0, 0),
                bias=self.b_qkv)
            y = sp.self_attention_gemm(xb, wf, vec, ops.LnFold(cs, stats, self.eps), self.w_nq, self.w_nk,
                                       self.rms_eps, cos, sin, B, L, H, hd, key_lens=_host_values(seq_lens))
        else:
            qkv = torch.empty((M, 3 * D), dtype=torch.bfloat16, device=dev)
            part = torch.empty((M, 2 * D // ops.RMS_BLOCK), dtype=torch.float32, device=dev) \
                if fused_exchange else None
            for sg in range(nseg):
                r0, r1 = (0, M) if nseg == 1 else (sg * L, (sg + 1) * L)
                b = sg if Be > 1 else 0  # modulation row of this segment
                if folds is not None:
                    wf, cs, vec = folds[2 * b]
                else:
                    wf, cs, vec = ops.fold_weight(self.w_qkv, mult_c=1.0, mult_a=mod[1], mult_b=e_row(b, 1),
                                                  shift_a=mod[0], shift_b=e_row(b, 0), bias=self.b_qkv)
                ln = ops.LnFold(cs, stats[r0:r1], self.eps)
                if fused_exchange:
                    ops.gemm_act(xb[r0:r1], wf, vec=vec, ln=ln, out=qkv[r0:r1], ms_out=part[r0:r1], ms_cols=2 * D)
                    continue
                seg_cos, seg_sin = (cos, sin) if sample_grids is None else \
                    self._rope_tables(sample_grids[sg], freqs, L)
                ops.gemm_norm(
                    xb[r0:r1], wf, vec=vec, ln=ln, norm_groups=2, norm_width=D,
                    norm_w=(self.w_nq, self.w_nk), norm_eps=self.rms_eps, rope_groups=2, rope_cos=seg_cos,
                    rope_sin=seg_sin, rows_per_batch=grid_rows_per_batch, token_offset=token_offset,
                    out=qkv[r0:r1], workspace=self.workspace,
                )
            if fused_exchange:
                y = sp.self_attention_p2p(qkv, part, self.w_nq, self.w_nk, self.rms_eps, cos, sin, B, L, H, hd,
                                          key_lens=_host_values(seq_lens))
            elif sp is not None:
                y = sp.self_attention(qkv, B, L, H, hd, key_lens=_host_values(seq_lens))
            else:
                q = qkv[:, :D].view(B, L, H, hd)
                k = qkv[:, D:2 * D].view(B, L, H, hd)
                v = qkv[:, 2 * D:].view(B, L, H, hd)
                y = local_attention(q, k, v, seq_lens).reshape(M, D)
        ops.gemm_residual(
            y, self.w_o, x32, out=x32, bias=self.b_o, gate_a=mod[2], gate_b=ev[:, 2 * D:], gate_b_stride=gate_stride,
            rows_per_batch=rows_per_batch, x_bf16_out=xb, stats_out=stats,
        )

        # --- cross-attention branch ---
        if self.cross_ln:
            cq = ops.gemm_norm(xb, self.w_cq, vec=self.vec_cq, ln=ops.LnFold(self.csum_cq, stats, self.cross_eps),
                               norm_groups=1, norm_width=D, norm_w=(self.w_cnq, None), norm_eps=self.rms_eps,
                               workspace=self.workspace)
        else:
            cq = ops.gemm_norm(xb, self.w_cq, vec=self.vec_cq, norm_groups=1, norm_width=D,
                               norm_w=(self.w_cnq, None), norm_eps=self.rms_eps, workspace=self.workspace)
        Bc, Lc, _ = context.shape
        pre_kv, self._pre_ckv = self._pre_ckv, None
        if pre_kv is not None and pre_kv[0] is context:
            ckv = pre_kv[1]
        else:
            ctx = context.reshape(Bc * Lc, D)
            if ctx.dtype != torch.bfloat16:
                ctx = ctx.to(torch.bfloat16)
            # split path: the same arithmetic as the model's all-blocks cross-K/V launch
            ckv = ops.gemm_norm(ctx, self.w_ckv, vec=self.b_ckv, norm_groups=1, norm_width=D,
                                norm_w=(self.w_cnk, None), norm_eps=self.rms_eps, workspace=self.workspace,
                                fused=False)
        ck = ckv[:, :D].view(Bc, Lc, H, hd)
        cv = ckv[:, D:].view(Bc, Lc, H, hd)
        cy = local_attention(cq.view(B, L, H, hd), ck, cv, context_lens).reshape(M, D)
        ops.gemm_residual(cy, self.w_co, x32, out=x32, bias=self.b_co, x_bf16_out=xb, stats_out=stats)

        # --- FFN branch ---
        h = torch.empty((M, self.ffn_dim), dtype=torch.bfloat16, device=dev)
        for b in range(Be):
            r0, r1 = (0, M) if Be == 1 else (b * L, (b + 1) * L)
            if folds is not None:
                wf, cs, vec = folds[2 * b + 1]
            else:
                wf, cs, vec = ops.fold_weight(self.w_1, mult_c=1.0, mult_a=mod[4], mult_b=e_row(b, 4),
                                              shift_a=mod[3], shift_b=e_row(b, 3), bias=self.b_1)
            timer = self.kernel_timer
            if timer is not None:
                ev0 = torch.cuda.Event(enable_timing=True)
                ev1 = torch.cuda.Event(enable_timing=True)
                ev0.record()
            ops.gemm_act(xb[r0:r1], wf, vec=vec, act="gelu_tanh", ln=ops.LnFold(cs, stats[r0:r1], self.eps),
                         out=h[r0:r1])
            if timer is not None:
                ev1.record()
                timer.append((ev0, ev1, 2.0 * (r1 - r0) * self.ffn_dim * D))
        ops.gemm_residual(
            h, self.w_2, x32, out=x32, bias=self.b_2, gate_a=mod[5], gate_b=ev[:, 5 * D:], gate_b_stride=gate_stride,
            rows_per_batch=rows_per_batch, x_bf16_out=xb, stats_out=stats,
        )
        # The residual epilogues wrote x32 in place through the C ABI: move its version so that
        # torch (and the carry key) see the change.
        torch.autograd.graph.increment_version(x32)
        self._carry().put(x32, xb, stats)
        return x32.view(B, L, D)

    # ------------------------------------------------------------------
    def alias_audit(self) -> dict:
        """Which packed operands share storage with the wrapped module's parameters
        (coda_wan/run_wan_coda.py:116-137)."""
        sa, ca = self.inner.self_attn, self.inner.cross_attn

        def same(a, b):
            return a.untyped_storage().data_ptr() == b.untyped_storage().data_ptr()

        checks = {
            "q_weight": same(sa.q.weight, self.w_qkv),
            "k_weight": same(sa.k.weight, self.w_qkv),
            "v_weight": same(sa.v.weight, self.w_qkv),
            "self_o_weight": same(sa.o.weight, self.w_o),
            "cross_kv_weight": same(ca.k.weight, self.w_ckv) and same(ca.v.weight, self.w_ckv),
            "cross_o_weight": same(ca.o.weight, self.w_co),
            "ffn1_weight": same(self.inner.ffn[0].weight, self.w_1),
            "ffn2_weight": same(self.inner.ffn[2].weight, self.w_2),
        }
        return {"checks": checks, "all_share_storage": all(checks.values())}


# Name used by the reference for the same drop-in.
CodaFullBlock = FusedWanBlock
