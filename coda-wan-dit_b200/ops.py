"""Fused ops of the Wan2.1 DiT block's non-attention half, on the wdit sm_100a kernels.

Two layers:

* Low-level fused GEMMs (``gemm_act``, ``gemm_residual``, ``gemm_norm``) and memory-bound
  passes (``ln_stats``, ``fold_weight``) with the full epilogue feature set; the drop-in
  block uses these. The model adds two all-blocks forms: ``fold_weight_batch`` (every adaLN
  weight fold of a step in one launch) and ``cross_kv_layers`` (every block's cross-attention
  K/V in one GEMM).
* The reference op API, same names / argument meaning / assertions as
  coda_wan/wan_coda_kernels.py and coda_wan/wan_gate_residual_coda.py:
  ``layernorm_modulation_bf16``, ``linear_bias_gelu_fixed``, ``qk_linear_bias_partial_rms``,
  ``qk_rms_rope_from_partials``, ``qk_coda_rms_rope``, ``rmsnorm_fused``,
  ``build_wan_rope_table``, ``prepack_linear_inplace``, ``prepack_qk_inplace``,
  ``replace_parameter_with_view``, ``unique_storage_bytes``,
  ``linear_gate_bias_residual_fixed``, ``linear_bias_residual_fixed``.

GEMM operand B is K-major ([N, K] = nn.Linear.weight). The reference passes ``b_kn`` (K, N);
its transposed view ``b_kn.t()`` is exactly that when ``b_kn`` is ``weight.T`` (what
``prepack_linear_inplace`` returns here). A contiguous (K, N) ``b_kn`` is transposed once.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from . import _lib
from ._lib import call, ptr, stream_ptr

DIM = 1536
HEAD_DIM = 128
RMS_BLOCK = 128
STATS_WIDTH = 256  # columns per LayerNorm-statistics partial (the GEMM's N tile)

_ACT = {"none": 0, "gelu_tanh": 1}


def _require_cuda(*ts: torch.Tensor | None) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("wdit ops run on CUDA tensors only (no CPU implementation)")


def _f32vec(v: torch.Tensor | None) -> torch.Tensor | None:
    if v is None:
        return None
    v = v.reshape(-1)
    if v.dtype != torch.float32:
        v = v.float()
    return v.contiguous()


def _rowmajor(t: torch.Tensor) -> torch.Tensor:
    """2-D with unit column stride (any row stride)."""
    assert t.dim() == 2
    if t.stride(1) != 1 or t.stride(0) < t.shape[1]:
        t = t.contiguous()
    return t


def _weight_nk(b_kn: torch.Tensor) -> torch.Tensor:
    """(K, N) operand -> [N, K] K-contiguous view (copy only if b_kn is N-major)."""
    w = b_kn.t()
    if w.stride(1) != 1:
        w = w.contiguous()
    return w


def stats_tiles(D: int) -> int:
    return (D + STATS_WIDTH - 1) // STATS_WIDTH


# ---------------------------------------------------------------------------
# Low-level fused GEMMs
# ---------------------------------------------------------------------------
class cta_pair:
    """Context manager selecting whether the tensor-bound GEMMs (``gemm_act``, long-K
    ``gemm_residual``) run on CTA pairs (256 x 256 tiles, the default) or on single CTAs."""

    def __init__(self, enable: bool):
        self.enable = bool(enable)
        self.prev = None

    def __enter__(self):
        self.prev = _lib.load().wdit_set_cta_pair(1 if self.enable else 0)
        return self

    def __exit__(self, *exc):
        _lib.load().wdit_set_cta_pair(self.prev)
        return False


class LnFold:
    """Absorbed LayerNorm: rstd_m * (acc - mu_m * csum[n]); (mu, rstd) from stats partials."""

    __slots__ = ("csum", "stats", "eps")

    def __init__(self, csum: torch.Tensor, stats: torch.Tensor, eps: float):
        self.csum = csum
        self.stats = stats
        self.eps = float(eps)


def _ln_args(ln: LnFold | None, K: int):
    if ln is None:
        return (None, None, 0, 0, 0.0)
    assert ln.csum.dtype == torch.float32 and ln.stats.dtype == torch.float32
    return (ptr(ln.csum), ptr(ln.stats), stats_tiles(K), STATS_WIDTH, ln.eps)


def gemm_act(a, w, *, vec=None, act="none", ln: LnFold | None = None, out=None, ms_out=None, ms_cols=0,
             max_ctas=0):
    """out[M,N] bf16 = act(LN(a @ w.T) + vec). a bf16 [M,K]; w bf16 [N,K].

    ms_out [M, >= ms_cols/128] fp32 (optional): mean of bf16(out)^2 over each 128-column block of
    the leading ms_cols columns (RMSNorm partials).
    """
    _require_cuda(a, w)
    a = _rowmajor(a)
    M, K = a.shape
    N = w.shape[0]
    assert w.shape[1] == K and w.stride(1) == 1
    assert a.dtype == torch.bfloat16 and w.dtype == torch.bfloat16
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=a.device)
    vec = _f32vec(vec)
    ms_ld = 0
    if ms_out is not None:
        assert ms_out.dtype == torch.float32 and ms_out.stride(1) == 1 and ms_out.shape[0] == M
        ms_ld = ms_out.stride(0)
    call(
        "wdit_gemm_act",
        ptr(a), a.stride(0), ptr(w), w.stride(0), ptr(out), out.stride(0), M, N, K,
        ptr(vec), _ACT[act], *_ln_args(ln, K), ptr(ms_out), ms_ld, ms_cols if ms_out is not None else 0,
        stream_ptr(), max_ctas,
    )
    return out


def gemm_residual(a, w, c, *, out=None, bias=None, gate_a=None, gate_b=None, gate_b_stride=0,
                  rows_per_batch=0, x_bf16_out=None, stats_out=None, max_ctas=0):
    """out[M,N] fp32 = c + (a @ w.T + bias) * (gate_a + gate_b[batch]); out may be c.

    gate_b is a raw [batches, gate_b_stride] fp32 view (per-batch modulation rows).
    """
    _require_cuda(a, w, c)
    a = _rowmajor(a)
    M, K = a.shape
    N = w.shape[0]
    assert w.shape[1] == K and w.stride(1) == 1
    assert c.dtype == torch.float32 and c.shape == (M, N) and c.stride(1) == 1
    if out is None:
        out = torch.empty_like(c)
    assert out.dtype == torch.float32 and out.shape == (M, N) and out.stride(1) == 1
    bias = _f32vec(bias)  # keep converted operands referenced until the launch is enqueued
    call(
        "wdit_gemm_residual",
        ptr(a), a.stride(0), ptr(w), w.stride(0), ptr(c), c.stride(0), ptr(out), out.stride(0), M, N, K,
        ptr(bias), ptr(gate_a), ptr(gate_b), gate_b_stride, rows_per_batch,
        ptr(x_bf16_out), 0 if x_bf16_out is None else x_bf16_out.stride(0), ptr(stats_out),
        stream_ptr(), max_ctas,
    )
    return out


def norm_workspace(M: int, N: int, norm_groups: int, norm_width: int, device) -> torch.Tensor:
    nbytes = int(_lib.load().wdit_gemm_norm_workspace_bytes(M, N, norm_groups, norm_width))
    return torch.empty(max(nbytes, 256), dtype=torch.uint8, device=device)


class Workspace:
    """Grow-only scratch for gemm_norm's RMSNorm partials (no initialization needed; launches
    on one stream may share it)."""

    def __init__(self):
        self.buf: torch.Tensor | None = None

    def get(self, M, N, groups, width, device) -> torch.Tensor:
        need = int(_lib.load().wdit_gemm_norm_workspace_bytes(M, N, groups, width))
        if self.buf is None or self.buf.numel() < need or self.buf.device != torch.device(device):
            self.buf = torch.empty(max(need, 256), dtype=torch.uint8, device=device)
        return self.buf


_default_ws: dict[int, Workspace] = {}


def _ws_for(device) -> Workspace:
    idx = torch.device(device).index or 0
    if idx not in _default_ws:
        _default_ws[idx] = Workspace()
    return _default_ws[idx]


def gemm_norm(a, w, *, vec=None, ln: LnFold | None = None, norm_groups=0, norm_width=0, norm_w=(None, None),
              norm_eps=1e-6, rope_groups=0, rope_cos=None, rope_sin=None, rows_per_batch=0, token_offset=0,
              out=None, workspace: Workspace | None = None, max_ctas=0, fused: bool | None = None):
    """out[M,N] bf16 = RoPE(RMSNorm_fullwidth(bf16(LN(a @ w.T) + vec))) per column group.

    rope_cos / rope_sin are token-major [T, 64] fp32 tables (row = token, column = rotary pair;
    any row stride that is a multiple of 4), as build_wan_rope_table returns them.

    fused: True = one launch with the RMSNorm / RoPE in the GEMM epilogue (wdit_gemm_norm_fused,
    no workspace; norm_width a multiple of 256); False / None (default) = the GEMM + partials,
    then the in-place RMSNorm / RoPE pass (wdit_gemm_norm, the reference's two-kernel split),
    which measures faster on B200 at the Wan shapes (QKV at M = 65520: 0.85 vs 0.93 ms).
    """
    _require_cuda(a, w)
    a = _rowmajor(a)
    M, K = a.shape
    N = w.shape[0]
    assert w.shape[1] == K and w.stride(1) == 1
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=a.device)
    fused = bool(fused) and norm_groups > 0
    ws = None
    nbytes = 0
    if norm_groups > 0 and not fused:
        ws = (workspace or _ws_for(a.device)).get(M, N, norm_groups, norm_width, a.device)
        nbytes = ws.numel()
    w0 = _f32vec(norm_w[0]) if norm_groups > 0 else None
    w1 = _f32vec(norm_w[1]) if norm_groups > 1 else None
    vec = _f32vec(vec)
    rope_ld = 0
    if rope_groups > 0:
        assert rope_cos.shape == rope_sin.shape and rope_cos.shape[1] == HEAD_DIM // 2
        assert rope_cos.dtype == torch.float32 and rope_sin.dtype == torch.float32
        assert rope_cos.stride(1) == 1 and rope_sin.stride() == rope_cos.stride()
        assert rope_cos.shape[0] >= (rows_per_batch or M) + token_offset, "RoPE tables shorter than the tokens"
        rope_ld = rope_cos.stride(0)
    if fused:
        call(
            "wdit_gemm_norm_fused",
            ptr(a), a.stride(0), ptr(w), w.stride(0), ptr(out), out.stride(0), M, N, K,
            ptr(vec), *_ln_args(ln, K), norm_groups, norm_width, ptr(w0), ptr(w1), float(norm_eps),
            rope_groups, ptr(rope_cos), ptr(rope_sin), rope_ld, rows_per_batch, token_offset,
            stream_ptr(), max_ctas,
        )
        return out
    call(
        "wdit_gemm_norm",
        ptr(a), a.stride(0), ptr(w), w.stride(0), ptr(out), out.stride(0), M, N, K,
        ptr(vec), *_ln_args(ln, K), norm_groups, norm_width, ptr(w0), ptr(w1), float(norm_eps),
        rope_groups, ptr(rope_cos), ptr(rope_sin), rope_ld, rows_per_batch, token_offset, ptr(ws), nbytes,
        stream_ptr(), max_ctas, kernels=2 if norm_groups > 0 else 1,
    )
    return out


def gemm_norm_exchange(a, w, *, vec, ln: LnFold | None, norm_w, norm_eps, rope_cos, rope_sin, batch, Lp, H, P,
                       rank, peers, full_off, flag_off, epoch, done_ctr, scratch=None, max_ctas=0):
    """Token-sharded QKV GEMM that delivers its output to the attention owners (wdit_gemm_norm_exchange).

    a [batch*Lp, K] this rank's tokens; w [3*H*128, K]; q and k get the full-width RMSNorm
    (weights norm_w) and the RoPE of their global tokens (rank*Lp + local token, tables with at
    least P*Lp rows); q, k, v land in full[3][U][P*Lp][128] of the rank owning each
    (batch, head) unit, in the exchange regions `peers` (ctypes array of P base addresses),
    and `epoch` is published into flags[rank] of every region when the launch is done.
    scratch [batch*Lp, 3*H*128] bf16 receives the pre-norm q / k (allocated when None).
    """
    _require_cuda(a, w)
    a = _rowmajor(a)
    M, K = a.shape
    N = w.shape[0]
    assert w.shape[1] == K and w.stride(1) == 1 and N == 3 * H * HEAD_DIM
    if scratch is None:
        scratch = torch.empty((M, N), dtype=torch.bfloat16, device=a.device)
    assert rope_cos.shape == rope_sin.shape and rope_cos.shape[1] == HEAD_DIM // 2
    assert rope_cos.dtype == torch.float32 and rope_sin.dtype == torch.float32
    assert rope_cos.stride(1) == 1 and rope_sin.stride() == rope_cos.stride()
    assert rope_cos.shape[0] >= P * Lp, "RoPE tables shorter than the sequence"
    call(
        "wdit_gemm_norm_exchange",
        ptr(a), a.stride(0), ptr(w), w.stride(0), ptr(scratch), scratch.stride(0), M, K,
        ptr(_f32vec(vec)), *_ln_args(ln, K), ptr(_f32vec(norm_w[0])), ptr(_f32vec(norm_w[1])), float(norm_eps),
        ptr(rope_cos), ptr(rope_sin), rope_cos.stride(0), batch, Lp, H, P, rank, peers, full_off, flag_off,
        epoch, done_ctr, stream_ptr(), max_ctas,
    )
    return scratch


def ln_stats(x, *, stats_out=None, x_bf16_out=None, x_f32_out=None):
    """Per-256-column (mean, M2) of the rows of x [M, D] (bf16 or fp32)."""
    _require_cuda(x)
    x = _rowmajor(x)
    M, D = x.shape
    if stats_out is None:
        stats_out = torch.empty((M, stats_tiles(D), 2), dtype=torch.float32, device=x.device)
    call(
        "wdit_ln_stats",
        ptr(x), 1 if x.dtype == torch.bfloat16 else 0, x.stride(0), M, D, ptr(stats_out), ptr(x_bf16_out),
        ptr(x_f32_out), stream_ptr(),
    )
    return stats_out


def fold_weight(w, *, mult_c, mult_a=None, mult_b=None, shift_a=None, shift_b=None, bias=None, w_out=None,
                csum_out=None, vec_out=None):
    """W'[n,k] = bf16(W[n,k] * (mult_c + mult_a[k] + mult_b[k])), csum = rowsum(W'),
    vec[n] = sum_k (shift_a + shift_b)[k] W[n,k] + bias[n]."""
    _require_cuda(w)
    N, K = w.shape
    assert w.stride(1) == 1 and w.dtype == torch.bfloat16
    if w_out is None:
        w_out = torch.empty((N, K), dtype=torch.bfloat16, device=w.device)
    if csum_out is None:
        csum_out = torch.empty(N, dtype=torch.float32, device=w.device)
    if vec_out is None:
        vec_out = torch.empty(N, dtype=torch.float32, device=w.device)
    bias = _f32vec(bias)
    call(
        "wdit_fold_weight",
        ptr(w), w.stride(0), N, K, float(mult_c), ptr(mult_a), ptr(mult_b), ptr(shift_a), ptr(shift_b),
        ptr(bias), ptr(w_out), w_out.stride(0), ptr(csum_out), ptr(vec_out), stream_ptr(),
    )
    return w_out, csum_out, vec_out


def patch_rows(latent: torch.Tensor, patch: tuple[int, int, int], token_lo: int, rows: int, Kp: int,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """Patch-embedding rows of latent [C, F, H, W]: out [rows, Kp] bf16, row r = the flattened
    (c, kt, kh, kw) patch of token token_lo + r (zero past the grid and past K columns)."""
    _require_cuda(latent)
    u = latent.to(torch.bfloat16).contiguous()
    C, F_, H, W = u.shape
    if out is None:
        out = torch.empty((rows, Kp), dtype=torch.bfloat16, device=u.device)
    assert out.shape == (rows, Kp) and out.is_contiguous() and out.dtype == torch.bfloat16
    call("wdit_patch_rows", ptr(u), C, F_, H, W, *patch, int(token_lo), rows, Kp, ptr(out), stream_ptr())
    return out


def cross_kv_layers(ctx: torch.Tensor, w_all: torch.Tensor, b_all: torch.Tensor, wk_all: torch.Tensor,
                    eps: float) -> torch.Tensor:
    """Cross-attention K and V of every block in one GEMM: ctx [M, D] bf16 times the blocks'
    packed [K_l; V_l] weights w_all [L * 2D, D] (+ b_all), then the WanRMSNorm of each K_l with
    weight wk_all[l] in one launch. Returns [M, L * 2D] bf16; block l's K and V are columns
    [2Dl, 2Dl + D) and [2Dl + D, 2D(l + 1)). Same arithmetic as `gemm_norm` per block."""
    L, D = wk_all.shape
    M = ctx.shape[0]
    N = w_all.shape[0]
    assert N == 2 * D * L and w_all.shape[1] == D and b_all.numel() == N and wk_all.stride(1) == 1
    part = torch.empty((M, N // RMS_BLOCK), dtype=torch.float32, device=ctx.device)
    out = gemm_act(ctx, w_all, vec=b_all, ms_out=part, ms_cols=N)
    call("wdit_rms_apply_layers", ptr(out), out.stride(0), M, ptr(part), part.stride(0), D, ptr(wk_all),
         float(eps), L, 2 * D, 2 * D // RMS_BLOCK, wk_all.stride(0), stream_ptr())
    return out


def fold_weight_batch(specs: list[dict]) -> list[tuple[torch.Tensor, torch.Tensor, torch.Tensor]]:
    """Many `fold_weight` calls in one launch. Each spec holds fold_weight's arguments
    (`w`, `mult_c`, optional `mult_a`, `mult_b`, `shift_a`, `shift_b`, `bias`); returns the
    (w_out, csum, vec) triple of each spec, in order."""
    if not specs:
        return []
    jobs = (_lib.FoldJob * len(specs))()
    outs, keep = [], []
    for j, sp in zip(jobs, specs):
        w = sp["w"]
        _require_cuda(w)
        N, K = w.shape
        assert w.stride(1) == 1 and w.dtype == torch.bfloat16
        w_out = torch.empty((N, K), dtype=torch.bfloat16, device=w.device)
        csum = torch.empty(N, dtype=torch.float32, device=w.device)
        vec = torch.empty(N, dtype=torch.float32, device=w.device)
        bias = _f32vec(sp.get("bias"))
        keep.append(bias)  # converted operands stay referenced until the launch is enqueued
        j.W, j.ldw, j.N, j.K, j.mult_c = ptr(w), w.stride(0), N, K, float(sp["mult_c"])
        j.mult_a, j.mult_b = ptr(sp.get("mult_a")), ptr(sp.get("mult_b"))
        j.shift_a, j.shift_b, j.bias = ptr(sp.get("shift_a")), ptr(sp.get("shift_b")), ptr(bias)
        j.W_out, j.ldw_out, j.csum_out, j.vec_out = ptr(w_out), w_out.stride(0), ptr(csum), ptr(vec)
        outs.append((w_out, csum, vec))
    launches = -(-len(specs) // _lib.FOLD_JOBS_PER_LAUNCH)
    call("wdit_fold_weight_batch", jobs, len(specs), stream_ptr(), kernels=launches)
    return outs


# ---------------------------------------------------------------------------
# Reference op API (coda_wan/wan_coda_kernels.py, coda_wan/wan_gate_residual_coda.py)
# ---------------------------------------------------------------------------
def layernorm_modulation_bf16(x: torch.Tensor, scale: torch.Tensor, shift: torch.Tensor, eps: float) -> torch.Tensor:
    """bf16(LN_noaffine(x) * (1 + scale) + shift).  wan_coda_kernels.py:59-81."""
    shape = x.shape
    x2 = x.reshape(-1, shape[-1])
    assert x2.shape[1] == DIM
    assert scale.numel() == shift.numel() == DIM
    _require_cuda(x2)
    x2 = _rowmajor(x2)
    out = torch.empty((x2.shape[0], DIM), dtype=torch.bfloat16, device=x.device)
    scale, shift = _f32vec(scale), _f32vec(shift)
    call(
        "wdit_layernorm_modulation",
        ptr(x2), 1 if x2.dtype == torch.bfloat16 else 0, x2.stride(0), x2.shape[0], DIM,
        ptr(scale), ptr(shift), float(eps), ptr(out), DIM, stream_ptr(),
    )
    return out.view(shape)


def linear_bias_gelu_fixed(a: torch.Tensor, b_kn: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """GELU-tanh(A @ B + bias) stored bf16.  wan_coda_kernels.py:120-152."""
    assert a.ndim == b_kn.ndim == 2 and bias.ndim == 1
    assert a.shape[1] == b_kn.shape[0] and b_kn.shape[1] == bias.shape[0]
    return gemm_act(a, _weight_nk(b_kn), vec=bias, act="gelu_tanh")


def qk_linear_bias_partial_rms(a, qk_weight_kn, qk_bias, block_size: int = RMS_BLOCK):
    """[q|k] = A @ W + b (bf16) and per-128-column mean-square partials [M, 24].
    wan_coda_kernels.py:192-230."""
    m, k = a.shape
    assert qk_weight_kn.shape == (k, 2 * DIM)
    assert qk_bias.shape == (2 * DIM,)
    assert (2 * DIM) % block_size == 0
    assert block_size == RMS_BLOCK, "partials are per 128-column block"
    partial = torch.empty((m, 2 * DIM // block_size), dtype=torch.float32, device=a.device)
    qk = gemm_act(a, _weight_nk(qk_weight_kn), vec=qk_bias, act="none", ms_out=partial, ms_cols=2 * DIM)
    return qk, partial


def qk_rms_rope_from_partials(qk, partial, q_weight, k_weight, cos, sin, eps):
    """WanRMSNorm (full width, bf16 roundings) + interleaved 3D RoPE, in place over qk.
    wan_coda_kernels.py:313-352."""
    m = qk.shape[0]
    assert qk.shape == (m, 2 * DIM)
    parts = DIM // RMS_BLOCK
    assert partial.shape == (m, 2 * parts)
    assert cos.shape == sin.shape == (m, HEAD_DIM // 2)
    _require_cuda(qk, partial, cos, sin)
    assert qk.stride(1) == 1 and partial.is_contiguous()
    wq, wk = _f32vec(q_weight), _f32vec(k_weight)
    cos, sin = cos.float().contiguous(), sin.float().contiguous()
    call(
        "wdit_qk_rms_rope_from_partials",
        ptr(qk), qk.stride(0), ptr(partial), m, DIM, ptr(wq), ptr(wk),
        ptr(cos), ptr(sin), float(eps), stream_ptr(),
    )
    return qk[:, :DIM], qk[:, DIM:]


def qk_coda_rms_rope(a, qk_weight_kn, qk_bias, q_weight, k_weight, cos, sin, eps):
    """One fused GEMM: q, k = RoPE(RMSNorm(A @ [Wq|Wk] + b)).  wan_coda_kernels.py:355-368.

    cos/sin are [m, 64] per-row tables (row i = token i), as in the reference.
    """
    m, k = a.shape
    assert qk_weight_kn.shape == (k, 2 * DIM)
    assert qk_bias.shape == (2 * DIM,)
    assert cos.shape == sin.shape == (m, HEAD_DIM // 2)
    qk = gemm_norm(
        a, _weight_nk(qk_weight_kn), vec=qk_bias, norm_groups=2, norm_width=DIM, norm_w=(q_weight, k_weight),
        norm_eps=eps, rope_groups=2, rope_cos=cos.float().contiguous(), rope_sin=sin.float().contiguous(),
        rows_per_batch=m, token_offset=0,
    )
    return qk[:, :DIM], qk[:, DIM:]


def rmsnorm_fused(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """bf16(bf16(x * rsqrt(mean(x^2) + eps)) * w) over the full width.  wan_coda_kernels.py:392-411."""
    shape = x.shape
    x2 = x.reshape(-1, shape[-1])
    assert x2.shape[1] == DIM
    _require_cuda(x2)
    x2 = _rowmajor(x2.to(torch.bfloat16) if x2.dtype != torch.bfloat16 else x2)
    out = torch.empty((x2.shape[0], DIM), dtype=torch.bfloat16, device=x.device)
    weight = _f32vec(weight)
    call("wdit_rmsnorm", ptr(x2), x2.stride(0), x2.shape[0], DIM, ptr(weight), float(eps), ptr(out), DIM,
         stream_ptr())
    return out.view(shape)


def _rope_table(grid_fhw, freqs: torch.Tensor, pair_major: bool):
    f, h, w = (int(v) for v in grid_fhw)
    _require_cuda(freqs)
    assert freqs.dim() == 2 and freqs.shape[1] == HEAD_DIM // 2 and freqs.is_complex()
    fr = torch.view_as_real(freqs.to(torch.complex128).contiguous()).contiguous()
    shape = (HEAD_DIM // 2, f * h * w) if pair_major else (f * h * w, HEAD_DIM // 2)
    cos = torch.empty(shape, dtype=torch.float32, device=freqs.device)
    sin = torch.empty_like(cos)
    call("wdit_rope_table", ptr(fr), freqs.shape[0], f, h, w, 1 if pair_major else 0, ptr(cos), ptr(sin),
         stream_ptr())
    return cos, sin


def build_wan_rope_table(grid_fhw, freqs: torch.Tensor):
    """Shared per-token cos/sin [f*h*w, 64] fp32 tables.  wan_coda_kernels.py:414-430."""
    return _rope_table(grid_fhw, freqs, pair_major=False)


def replace_parameter_with_view(module: nn.Module, name: str, view: torch.Tensor) -> None:
    module._parameters[name] = nn.Parameter(view, requires_grad=False)


def prepack_linear_inplace(linear: nn.Linear) -> torch.Tensor:
    """(K, N) operand of a Linear with zero copies: the K-major weight is the GEMM's native
    B layout, so the packed operand is a transposed view of the parameter's own storage.
    Counterpart of wan_coda_kernels.py:441-445 (which needs a transpose copy for its GEMM)."""
    return linear.weight.detach().T


def prepack_qk_inplace(q: nn.Linear, k: nn.Linear):
    """Pack Q and K into one [2N, K] allocation; the parameters become views of it.
    wan_coda_kernels.py:448-461."""
    packed = torch.cat([q.weight.detach(), k.weight.detach()], dim=0).contiguous()
    bias = torch.cat([q.bias.detach(), k.bias.detach()]).contiguous()
    n = q.weight.shape[0]
    replace_parameter_with_view(q, "weight", packed[:n])
    replace_parameter_with_view(k, "weight", packed[n:])
    replace_parameter_with_view(q, "bias", bias[:n])
    replace_parameter_with_view(k, "bias", bias[n:])
    return packed.T, bias


def prepack_qkv_inplace(q: nn.Linear, k: nn.Linear, v: nn.Linear):
    """Q, K and V packed into one [3N, K] allocation (the fused QKV GEMM's B operand);
    the three Linear parameters become views of it (no duplicate bytes)."""
    packed = torch.cat([q.weight.detach(), k.weight.detach(), v.weight.detach()], dim=0).contiguous()
    bias = torch.cat([q.bias.detach(), k.bias.detach(), v.bias.detach()]).contiguous()
    n = q.weight.shape[0]
    for i, lin in enumerate((q, k, v)):
        replace_parameter_with_view(lin, "weight", packed[i * n:(i + 1) * n])
        replace_parameter_with_view(lin, "bias", bias[i * n:(i + 1) * n])
    return packed, bias


def unique_storage_bytes(module: nn.Module, extras: list[torch.Tensor]) -> int:
    """Unique CUDA storage bytes across parameters, buffers and extras.  wan_coda_kernels.py:464-477."""
    seen: set[tuple[int, int]] = set()
    total = 0
    for tensor in list(module.parameters()) + list(module.buffers()) + list(extras):
        if tensor.device.type != "cuda":
            continue
        storage = tensor.untyped_storage()
        key = (storage.data_ptr(), storage.nbytes())
        if key not in seen:
            seen.add(key)
            total += storage.nbytes()
    return total


def linear_gate_bias_residual_fixed(A, B, C, gate, bias, *, inplace: bool = False):
    """(A @ B) * gate + bias * gate + C in fp32; out may alias C.  wan_gate_residual_coda.py:192-242."""
    assert gate.shape == bias.shape == (B.shape[1],)
    assert A.ndim == B.ndim == C.ndim == 2
    out = C if inplace else torch.empty_like(C)
    return gemm_residual(A, _weight_nk(B), C, out=out, bias=bias, gate_a=_f32vec(gate))


def linear_bias_residual_fixed(A, B, C, bias, *, inplace: bool = False):
    """A @ B + bias + C in fp32; out may alias C.  wan_gate_residual_coda.py:99-135."""
    assert A.ndim == B.ndim == C.ndim == 2
    assert bias.shape == (B.shape[1],)
    assert A.shape[0] == C.shape[0] and B.shape[1] == C.shape[1]
    out = C if inplace else torch.empty_like(C)
    return gemm_residual(A, _weight_nk(B), C, out=out, bias=bias)
