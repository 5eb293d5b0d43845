"""Per-op oracle: the reference's fused-op arithmetic restated in PyTorch (fp32 math).

Test infrastructure only (see oracle/__init__.py). Each function cites the reference
(Owen718/CODA-Wan-DiT) code it restates. The GEMM-epilogue ops of the reference run on an
absent sm_90 GEMM (coda-kernels `rapier`); their epilogue math is explicit in the
reference's EVT classes and is restated here on top of an fp32 matmul of the bf16 operands.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

DIM = 1536
HEAD_DIM = 128
RMS_BLOCK = 128
GELU_C0 = 0.7978845608028654  # coda_wan/wan_coda_kernels.py:100
GELU_C1 = 0.044715            # coda_wan/wan_coda_kernels.py:100
STATS_WIDTH = 256


def to_bf16(x: torch.Tensor, mode: str = "rne") -> torch.Tensor:
    """fp32 -> bf16 with round-to-nearest-even ("rne", CUDA / GPU Triton semantics) or
    round-toward-zero ("rz": what Triton's CPU interpreter does, which the golden fixtures made
    with it carry)."""
    x = x.float()
    if mode == "rne":
        return x.to(torch.bfloat16)
    if mode == "rz":
        return (x.contiguous().view(torch.int32) & ~0xFFFF).view(torch.float32).to(torch.bfloat16)
    raise ValueError(mode)


def bf16r(x: torch.Tensor, mode: str = "rne") -> torch.Tensor:
    """Round to bf16 and back to fp32."""
    return to_bf16(x, mode).float()


def mm_f32(a: torch.Tensor, b_kn: torch.Tensor) -> torch.Tensor:
    """fp32 product of bf16 operands (the tensor-core contraction with fp32 accumulation)."""
    return a.float() @ b_kn.float()


def gelu_tanh(x: torch.Tensor) -> torch.Tensor:
    """coda_wan/wan_coda_kernels.py:99-101 (EVTGELUBias.consumer_visit)."""
    z = GELU_C0 * (x + GELU_C1 * x * x * x)
    return 0.5 * x * (1.0 + torch.tanh(z))


def layernorm_modulation(x: torch.Tensor, scale: torch.Tensor, shift: torch.Tensor, eps: float,
                         mode: str = "rne") -> torch.Tensor:
    """bf16((x - mean) * rsqrt(var + eps) * (1 + scale) + shift), biased variance, fp32.
    coda_wan/wan_coda_kernels.py:45-56."""
    x = x.float()
    mean = x.mean(-1, keepdim=True)
    c = x - mean
    var = (c * c).mean(-1, keepdim=True)
    y = c * torch.rsqrt(var + eps)
    return to_bf16(y * (1.0 + scale.float()) + shift.float(), mode)


def linear_bias_gelu(a: torch.Tensor, b_kn: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """bf16(gelu_tanh(A @ B + bias)).  coda_wan/wan_coda_kernels.py:84-152."""
    return gelu_tanh(mm_f32(a, b_kn) + bias.float()).to(torch.bfloat16)


def qk_linear_bias_partial_rms(a, qk_weight_kn, qk_bias, block_size=RMS_BLOCK):
    """qk = bf16(A @ W + b); partial[m, j] = mean over column block j of qk^2.
    coda_wan/wan_coda_kernels.py:155-230 (EVTRowOrColBias + EVTColBlockReductionStore with the
    mean-square op, inv_block_size = 1/tile_N). The partial is taken here over the stored bf16
    values, the quantity WanRMSNorm normalizes."""
    acc = mm_f32(a, qk_weight_kn) + qk_bias.float()
    qk = acc.to(torch.bfloat16)
    m, n = qk.shape
    partial = qk.float().square().view(m, n // block_size, block_size).mean(-1)
    return qk, partial


def qk_rms_rope_from_partials(qk, partial, q_weight, k_weight, cos, sin, eps, mode: str = "rne"):
    """coda_wan/wan_coda_kernels.py:233-352 restated: rstd from the mean of the 12 partials of
    each half, y = bf16(bf16(x * rstd) * w), then interleaved-pair RoPE in fp32 with the
    per-token table row pair = (d % 128) // 2, stored bf16. Returns new (q, k) tensors."""
    m = qk.shape[0]
    parts = DIM // RMS_BLOCK
    outs = []
    for half, w in ((0, q_weight), (1, k_weight)):
        x = qk[:, half * DIM:(half + 1) * DIM].float()
        ms = partial[:, half * parts:(half + 1) * parts].float().sum(-1, keepdim=True) / parts
        rstd = torch.rsqrt(ms + eps)
        y = bf16r(x * rstd, mode)
        y = bf16r(y * w.float(), mode)
        y = y.view(m, DIM // 2, 2)
        pair = (torch.arange(DIM // 2, device=qk.device) % (HEAD_DIM // 2))
        c = cos.float()[:, pair]
        s = sin.float()[:, pair]
        e, o = y[..., 0], y[..., 1]
        out = torch.stack([e * c - o * s, e * s + o * c], dim=-1).reshape(m, DIM)
        outs.append(to_bf16(out, mode))
    return outs[0], outs[1]


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, mode: str = "rne") -> torch.Tensor:
    """bf16(bf16(x * rsqrt(mean(x^2) + eps)) * w).  coda_wan/wan_coda_kernels.py:371-411."""
    xf = x.float()
    y = bf16r(xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + eps), mode)
    return to_bf16(y * w.float(), mode)


def build_wan_rope_table(grid_fhw, freqs):
    """coda_wan/wan_coda_kernels.py:414-430 restated: cos/sin fp32 [f*h*w, 64]."""
    f, h, w = grid_fhw
    c = HEAD_DIM // 2
    n1 = c - 2 * (c // 3)
    parts = (freqs[:, :n1], freqs[:, n1:n1 + c // 3], freqs[:, n1 + c // 3:])
    tab = torch.cat(
        [
            parts[0][:f].view(f, 1, 1, -1).expand(f, h, w, -1),
            parts[1][:h].view(1, h, 1, -1).expand(f, h, w, -1),
            parts[2][:w].view(1, 1, w, -1).expand(f, h, w, -1),
        ],
        dim=-1,
    ).reshape(f * h * w, c)
    return tab.real.float().contiguous(), tab.imag.float().contiguous()


def linear_gate_bias_residual(A, B, C, gate, bias):
    """(A @ B) * g + (b * g) + C in fp32.  coda_wan/wan_gate_residual_coda.py:138-161, 192-242."""
    g = gate.float()
    return mm_f32(A, B) * g + bias.float() * g + C.float()


def linear_bias_residual(A, B, C, bias):
    """A @ B + bias + C in fp32.  coda_wan/wan_gate_residual_coda.py:75-135."""
    return mm_f32(A, B) + bias.float() + C.float()


# ---------------------------------------------------------------------------
# The build's fused formulations (the algebra the kernels implement), for op-level checks
# ---------------------------------------------------------------------------
def ln_stats(x: torch.Tensor, width: int = STATS_WIDTH) -> torch.Tensor:
    """Per-`width`-column (mean, M2) of each row: [M, ceil(D/width), 2] fp32."""
    x = x.float()
    M, D = x.shape
    out = []
    for c0 in range(0, D, width):
        seg = x[:, c0:c0 + width]
        mean = seg.mean(-1)
        m2 = (seg - mean[:, None]).square().sum(-1)
        out.append(torch.stack([mean, m2], dim=-1))
    return torch.stack(out, dim=1)


def merge_stats(stats: torch.Tensor, D: int, eps: float, width: int = STATS_WIDTH):
    """(mu, rstd) per row from (mean, M2) partials (Chan's parallel merge)."""
    n_t = torch.tensor([min(width, D - t * width) for t in range(stats.shape[1])], dtype=torch.float64,
                       device=stats.device)
    mean_t = stats[..., 0].double()
    m2_t = stats[..., 1].double()
    mu = (mean_t * n_t).sum(-1) / D
    m2 = m2_t.sum(-1) + ((mean_t - mu[:, None]).square() * n_t).sum(-1)
    return mu.float(), torch.rsqrt(m2 / D + eps).float()


def fold_weight(w_nk, mult, shift, bias):
    """W' = bf16(W * mult[k]); csum[n] = sum_k W'[n,k]; vec[n] = sum_k shift[k] W[n,k] + bias[n]."""
    wf = bf16r(w_nk.float() * mult.float()[None, :])
    csum = wf.sum(-1)
    vec = (w_nk.float() * shift.float()[None, :]).sum(-1) + (bias.float() if bias is not None else 0.0)
    return wf.to(torch.bfloat16), csum, vec


def ln_folded_matmul(x_bf16, w_fold_nk, csum, vec, stats, eps):
    """rstd * (x @ W'^T - mu * csum) + vec (the absorbed LayerNorm + modulation)."""
    mu, rstd = merge_stats(stats, x_bf16.shape[1], eps)
    acc = x_bf16.float() @ w_fold_nk.float().t()
    return rstd[:, None] * (acc - mu[:, None] * csum[None, :]) + vec[None, :]


def rope_rows(y: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Interleaved-pair rotation of y [M, W] (W a multiple of 128) by per-row cos/sin [M, 64]."""
    M, W = y.shape
    pair = torch.arange(W // 2, device=y.device) % (HEAD_DIM // 2)
    c = cos[:, pair]
    s = sin[:, pair]
    v = y.view(M, W // 2, 2)
    e, o = v[..., 0], v[..., 1]
    return torch.stack([e * c - o * s, e * s + o * c], dim=-1).reshape(M, W)


def norm_epilogue(acc, norm_groups, width, norm_w, eps, rope_groups=0, cos=None, sin=None):
    """bf16 projection -> full-width WanRMSNorm per column group -> RoPE -> bf16."""
    y = bf16r(acc)
    out = y.clone()
    for g in range(norm_groups):
        seg = y[:, g * width:(g + 1) * width]
        rstd = torch.rsqrt(seg.square().mean(-1, keepdim=True) + eps)
        z = bf16r(bf16r(seg * rstd) * norm_w[g].float()[None, :])
        if g < rope_groups:
            z = rope_rows(z, cos, sin)
        out[:, g * width:(g + 1) * width] = z
    return out.to(torch.bfloat16)


def sdpa(q, k, v):
    """q [B, Lq, H, hd] ... fp32 attention (no mask)."""
    return F.scaled_dot_product_attention(q.float().transpose(1, 2), k.float().transpose(1, 2),
                                          v.float().transpose(1, 2)).transpose(1, 2)
