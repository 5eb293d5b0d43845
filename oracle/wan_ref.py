"""Stock Wan2.1 DiT restated in eager PyTorch: the oracle the fused path must match.

Test infrastructure only (see oracle/__init__.py). Runs on CPU in fp32 (config 0) and on a
GPU in fp32 or in the stock bf16 mixed precision (Linear / attention in bf16, residual
stream, modulation, LayerNorm and RoPE in fp32 or wider).

Sources of the math (the upstream Wan2.1 package is not installed, so nothing here is taken
from its source; each piece is restated from the formula):
  block          coda_wan/docs/report.md:37-43, docs/walkthrough.md:27-32:
                   e = (modulation + e0).chunk(6)
                   x = x + self_attn(norm1(x)(1+e1) + e0) * e2
                   x = x + cross_attn(norm3(x), context)
                   x = x + ffn(norm2(x)(1+e4) + e3) * e5
  numerics       as encoded by the reference's fused path: fp32 modulation add
                 (coda_wan/run_wan_coda.py:142), affine-free LayerNorm eps 1e-6 in fp32
                 (coda_wan/wan_coda_kernels.py:49-55), WanRMSNorm over the full width with a
                 rounding to the activation dtype before the weight (:284-288, :386-388),
                 interleaved-pair 3D RoPE with the [22, 21, 21] complex-column split and
                 theta 1e4 (:414-430, :290-300) applied in float64 as stock Wan does,
                 tanh-GELU (:100-101), gate multiply and residual add in fp32
                 (coda_wan/wan_gate_residual_coda.py:201-214), affine norm3
                 (coda_wan/run_wan_coda.py:176), cross RMSNorm on q and k only (:177-183).
  model parts    patch embedding Conv3d(16 -> dim, kernel = stride = (1, 2, 2)), text MLP
                 4096 -> dim -> dim with tanh-GELU, sinusoidal time embedding (256) ->
                 Linear-SiLU-Linear, SiLU-Linear to 6*dim, head LayerNorm + 2-vector
                 modulation + Linear(dim -> 64), unpatchify. UNVERIFIED vs upstream.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass(frozen=True)
class WanConfig:
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
    cross_attn_norm: bool = True

    @property
    def head_dim(self) -> int:
        return self.dim // self.num_heads


WAN_1_3B = WanConfig()
WAN_14B = WanConfig(dim=5120, ffn_dim=13824, num_heads=40, num_layers=40)


# ---------------------------------------------------------------------------
# Numerics helpers
# ---------------------------------------------------------------------------
def linear(mod: nn.Linear, x: torch.Tensor, cd: torch.dtype) -> torch.Tensor:
    """Linear in the compute dtype (bf16 under the stock mixed precision)."""
    b = mod.bias.to(cd) if mod.bias is not None else None
    return F.linear(x.to(cd), mod.weight.to(cd), b)


def gelu_tanh(x: torch.Tensor) -> torch.Tensor:
    return F.gelu(x, approximate="tanh")


class RMSNormRef(nn.Module):
    """WanRMSNorm semantics: normalize in fp32 over the full width, round to the input
    dtype, then multiply by the weight (coda_wan/wan_coda_kernels.py:284-288)."""

    def __init__(self, dim: int, eps: float):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        xf = x.float()
        y = xf * torch.rsqrt(xf.square().mean(dim=-1, keepdim=True) + self.eps)
        return y.to(x.dtype) * self.weight.to(x.dtype)


class LayerNormRef(nn.Module):
    """LayerNorm computed in fp32 (optionally affine), returned in the input dtype."""

    def __init__(self, dim: int, eps: float, affine: bool):
        super().__init__()
        self.dim = dim
        self.eps = eps
        if affine:
            self.weight = nn.Parameter(torch.ones(dim))
            self.bias = nn.Parameter(torch.zeros(dim))
        else:
            self.register_parameter("weight", None)
            self.register_parameter("bias", None)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        w = self.weight.float() if self.weight is not None else None
        b = self.bias.float() if self.bias is not None else None
        return F.layer_norm(x.float(), (self.dim,), w, b, self.eps).to(x.dtype)


def rope_freqs(max_pos: int, head_dim: int, theta: float = 10000.0) -> torch.Tensor:
    """complex128 [max_pos, head_dim/2]: per-axis rotary frequencies, the head dimension
    split 44/42/42 (frame/height/width) for head_dim 128: d - 4(d//6), 2(d//6), 2(d//6)."""
    d = head_dim
    dims = [d - 4 * (d // 6), 2 * (d // 6), 2 * (d // 6)]
    parts = []
    for n in dims:
        inv = 1.0 / torch.pow(torch.tensor(theta, dtype=torch.float64), torch.arange(0, n, 2, dtype=torch.float64) / n)
        ang = torch.outer(torch.arange(max_pos, dtype=torch.float64), inv)
        parts.append(torch.polar(torch.ones_like(ang), ang))
    return torch.cat(parts, dim=1)


def rope_table(grid: tuple[int, int, int], freqs: torch.Tensor) -> torch.Tensor:
    """complex [f*h*w, 64] per-token rotation: columns [0,22) from the frame index,
    [22,43) from the row index, [43,64) from the column index."""
    f, h, w = grid
    c = freqs.shape[1]
    n1 = c - 2 * (c // 3)
    n2 = c // 3
    fr, hr, wr = freqs[:, :n1], freqs[:, n1:n1 + n2], freqs[:, n1 + n2:]
    tab = torch.cat(
        [
            fr[:f].view(f, 1, 1, -1).expand(f, h, w, -1),
            hr[:h].view(1, h, 1, -1).expand(f, h, w, -1),
            wr[:w].view(1, 1, w, -1).expand(f, h, w, -1),
        ],
        dim=-1,
    )
    return tab.reshape(f * h * w, c)


def rope_apply(x: torch.Tensor, grids: list[tuple[int, int, int]], freqs: torch.Tensor) -> torch.Tensor:
    """x [B, L, H, hd]; rotate interleaved pairs (2i, 2i+1) of the first f*h*w tokens of each
    sample in float64; returns fp32."""
    B, L, H, hd = x.shape
    out = x.float().clone()
    for i in range(B):
        f, h, w = grids[i]
        n = f * h * w
        tab = rope_table((f, h, w), freqs.to(x.device)).view(n, 1, hd // 2)
        xc = torch.view_as_complex(x[i, :n].to(torch.float64).reshape(n, H, hd // 2, 2))
        out[i, :n] = torch.view_as_real(xc * tab).reshape(n, H, hd).float()
    return out


def _host_list(v):
    """Python values of a small tensor / sequence (no device-side compute)."""
    return v.tolist() if torch.is_tensor(v) else list(v)


def attention(q, k, v, k_lens, cd):
    """q [B, Lq, H, hd], k/v [B, Lk, H, hd]; softmax(q k^T / sqrt(hd)) v with keys >= k_lens masked."""
    B, Lq, H, hd = q.shape
    Lk = k.shape[1]
    mask = None
    if k_lens is not None:
        lens = _host_list(k_lens)
        if any(int(v) < Lk for v in lens):
            kl = torch.tensor([int(v) for v in lens], device=q.device).view(B, 1, 1, 1)
            mask = torch.arange(Lk, device=q.device).view(1, 1, 1, Lk) < kl
    o = F.scaled_dot_product_attention(
        q.to(cd).transpose(1, 2), k.to(cd).transpose(1, 2), v.to(cd).transpose(1, 2), attn_mask=mask
    )
    return o.transpose(1, 2)


# ---------------------------------------------------------------------------
# Block
# ---------------------------------------------------------------------------
class SelfAttentionRef(nn.Module):
    def __init__(self, dim, num_heads, eps):
        super().__init__()
        self.dim = dim
        self.num_heads = num_heads
        self.head_dim = dim // num_heads
        self.eps = eps
        self.window_size = (-1, -1)
        self.q = nn.Linear(dim, dim)
        self.k = nn.Linear(dim, dim)
        self.v = nn.Linear(dim, dim)
        self.o = nn.Linear(dim, dim)
        self.norm_q = RMSNormRef(dim, eps)
        self.norm_k = RMSNormRef(dim, eps)

    def forward(self, x, seq_lens, grids, freqs, cd):
        B, L, _ = x.shape
        H, hd = self.num_heads, self.head_dim
        q = self.norm_q(linear(self.q, x, cd)).view(B, L, H, hd)
        k = self.norm_k(linear(self.k, x, cd)).view(B, L, H, hd)
        v = linear(self.v, x, cd).view(B, L, H, hd)
        q = rope_apply(q, grids, freqs)
        k = rope_apply(k, grids, freqs)
        y = attention(q, k, v, seq_lens, cd)
        return linear(self.o, y.reshape(B, L, self.dim), cd)


class CrossAttentionRef(SelfAttentionRef):
    def forward(self, x, context, context_lens, cd):
        B, L, _ = x.shape
        Lc = context.shape[1]
        H, hd = self.num_heads, self.head_dim
        q = self.norm_q(linear(self.q, x, cd)).view(B, L, H, hd)
        k = self.norm_k(linear(self.k, context, cd)).view(B, Lc, H, hd)
        v = linear(self.v, context, cd).view(B, Lc, H, hd)
        y = attention(q, k, v, context_lens, cd)
        return linear(self.o, y.reshape(B, L, self.dim), cd)


class WanBlockRef(nn.Module):
    """Stock Wan attention block (eager). forward(x, e, seq_lens, grid_sizes, freqs, context,
    context_lens) -> x (fp32)."""

    def __init__(self, cfg: WanConfig, compute_dtype: torch.dtype = torch.float32):
        super().__init__()
        d = cfg.dim
        self.dim = d
        self.ffn_dim = cfg.ffn_dim
        self.num_heads = cfg.num_heads
        self.window_size = (-1, -1)
        self.eps = cfg.eps
        self.compute_dtype = compute_dtype
        self.norm1 = LayerNormRef(d, cfg.eps, affine=False)
        self.self_attn = SelfAttentionRef(d, cfg.num_heads, cfg.eps)
        self.norm3 = LayerNormRef(d, cfg.eps, affine=True) if cfg.cross_attn_norm else nn.Identity()
        self.cross_attn = CrossAttentionRef(d, cfg.num_heads, cfg.eps)
        self.norm2 = LayerNormRef(d, cfg.eps, affine=False)
        self.ffn = nn.Sequential(nn.Linear(d, cfg.ffn_dim), nn.GELU(approximate="tanh"), nn.Linear(cfg.ffn_dim, d))
        self.modulation = nn.Parameter(torch.randn(1, 6, d) / d**0.5)

    def forward(self, x, e, seq_lens, grid_sizes, freqs, context, context_lens):
        cd = self.compute_dtype
        grids = [tuple(int(v) for v in g) for g in _host_list(grid_sizes)]
        e = (self.modulation.float() + e.float()).chunk(6, dim=1)
        y = self.self_attn(self.norm1(x).float() * (1 + e[1]) + e[0], seq_lens, grids, freqs, cd)
        x = x + y * e[2]
        x = x + self.cross_attn(self.norm3(x), context, context_lens, cd)
        h = gelu_tanh(linear(self.ffn[0], self.norm2(x).float() * (1 + e[4]) + e[3], cd))
        y = linear(self.ffn[2], h, cd)
        x = x + y * e[5]
        return x


# ---------------------------------------------------------------------------
# Model (non-block parts UNVERIFIED vs upstream)
# ---------------------------------------------------------------------------
def sinusoidal_embedding(dim: int, pos: torch.Tensor) -> torch.Tensor:
    half = dim // 2
    p = pos.to(torch.float64)
    freq = torch.pow(10000.0, -torch.arange(half, dtype=torch.float64, device=p.device) / half)
    s = torch.outer(p, freq)
    return torch.cat([torch.cos(s), torch.sin(s)], dim=1)


class HeadRef(nn.Module):
    def __init__(self, cfg: WanConfig):
        super().__init__()
        d = cfg.dim
        self.out_features = math.prod(cfg.patch) * cfg.out_dim
        self.norm = LayerNormRef(d, cfg.eps, affine=False)
        self.head = nn.Linear(d, self.out_features)
        self.modulation = nn.Parameter(torch.randn(1, 2, d) / d**0.5)

    def forward(self, x, e, cd):
        e2 = (self.modulation.float() + e.float().unsqueeze(1)).chunk(2, dim=1)
        return linear(self.head, self.norm(x).float() * (1 + e2[1]) + e2[0], cd)


class WanModelRef(nn.Module):
    def __init__(self, cfg: WanConfig = WAN_1_3B, compute_dtype: torch.dtype = torch.float32,
                 num_layers: int | None = None):
        super().__init__()
        self.cfg = cfg
        d = cfg.dim
        self.dim = d
        self.num_heads = cfg.num_heads
        self.compute_dtype = compute_dtype
        self.patch_embedding = nn.Conv3d(cfg.in_dim, d, kernel_size=cfg.patch, stride=cfg.patch)
        self.text_embedding = nn.Sequential(nn.Linear(cfg.text_dim, d), nn.GELU(approximate="tanh"), nn.Linear(d, d))
        self.time_embedding = nn.Sequential(nn.Linear(cfg.freq_dim, d), nn.SiLU(), nn.Linear(d, d))
        self.time_projection = nn.Sequential(nn.SiLU(), nn.Linear(d, 6 * d))
        n = cfg.num_layers if num_layers is None else num_layers
        self.blocks = nn.ModuleList([WanBlockRef(cfg, compute_dtype) for _ in range(n)])
        self.head = HeadRef(cfg)
        self.register_buffer("freqs", rope_freqs(1024, cfg.head_dim), persistent=False)

    def embed(self, x_list, t, context_list, seq_len):
        cd = self.compute_dtype
        cfg = self.cfg
        xs = [F.conv3d(u.unsqueeze(0).to(cd), self.patch_embedding.weight.to(cd), self.patch_embedding.bias.to(cd),
                       stride=cfg.patch) for u in x_list]
        grids = [tuple(int(d) for d in u.shape[2:]) for u in xs]
        xs = [u.flatten(2).transpose(1, 2) for u in xs]
        seq_lens = [int(u.shape[1]) for u in xs]
        x = torch.cat([torch.cat([u, u.new_zeros(1, seq_len - u.shape[1], u.shape[2])], dim=1) for u in xs])
        tt = torch.as_tensor(t, device=x.device).reshape(-1)
        e = self.time_embedding.float()(sinusoidal_embedding(cfg.freq_dim, tt).float())
        e0 = self.time_projection.float()(e).unflatten(1, (6, self.dim))
        ctx = torch.stack([torch.cat([u, u.new_zeros(cfg.text_len - u.shape[0], u.shape[1])]) for u in context_list])
        c = gelu_tanh(linear(self.text_embedding[0], ctx, cd))
        context = linear(self.text_embedding[2], c, cd)
        return x, e, e0, seq_lens, grids, context

    def unpatchify(self, x, grids):
        cfg = self.cfg
        outs = []
        for u, (f, h, w) in zip(x, grids):
            n = f * h * w
            u = u[:n].view(f, h, w, *cfg.patch, cfg.out_dim)
            u = torch.einsum("fhwpqrc->cfphqwr", u)
            outs.append(u.reshape(cfg.out_dim, f * cfg.patch[0], h * cfg.patch[1], w * cfg.patch[2]))
        return outs

    def forward(self, x_list, t, context_list, seq_len):
        x, e, e0, seq_lens, grids, context = self.embed(x_list, t, context_list, seq_len)
        for blk in self.blocks:
            x = blk(x, e0, seq_lens, grids, self.freqs, context, None)
        x = self.head(x, e, self.compute_dtype)
        return [u.float() for u in self.unpatchify(x, grids)]


# ---------------------------------------------------------------------------
# Seeded initialisation and inputs
# ---------------------------------------------------------------------------
def init_weights_(module: nn.Module, seed: int, norm_jitter: float = 0.0) -> nn.Module:
    """Linear / conv weights ~N(0, 0.02), biases ~N(0, 0.01), modulation ~N(0,1)/sqrt(dim);
    norm weights 1 (norm_jitter > 0 perturbs them, and norm3's bias, to exercise the folds).
    The generator lives on the parameters' device (a module built on a GPU is initialised there;
    its values then differ from a CPU-initialised one with the same seed)."""
    first = next(module.parameters(), None)
    dev = first.device if first is not None else torch.device("cpu")
    g = torch.Generator(device=dev).manual_seed(seed)

    def randn(shape):
        return torch.randn(shape, generator=g, device=dev)

    with torch.no_grad():
        for name, p in module.named_parameters():
            leaf = name.rsplit(".", 1)[-1]
            if "modulation" in name:
                p.copy_(randn(p.shape) / p.shape[-1] ** 0.5)
            elif "norm" in name:
                if leaf == "weight":
                    p.copy_(1.0 + norm_jitter * randn(p.shape))
                else:
                    p.copy_(norm_jitter * randn(p.shape))
            elif leaf == "weight":
                p.copy_(0.02 * randn(p.shape))
            elif leaf == "bias":
                p.copy_(0.01 * randn(p.shape))
    return module


def model_on_device(cfg: WanConfig, compute_dtype: torch.dtype, device, seed: int,
                    num_layers: int | None = None) -> "WanModelRef":
    """A WanModelRef built directly on `device` (no CPU copy of the weights) and initialised
    there with init_weights_ (fp32 parameters, the rotary frequencies in complex128)."""
    with torch.device("meta"):
        m = WanModelRef(cfg, compute_dtype, num_layers=num_layers)
    m = m.to_empty(device=device)
    m.freqs = rope_freqs(1024, cfg.head_dim).to(device)
    return init_weights_(m, seed)


def block_inputs(cfg: WanConfig, grid: tuple[int, int, int], batch: int, seed: int, ctx_len: int = 512,
                 device="cpu", x_dtype=torch.float32):
    """Config 0/1 inputs: x ~N(0,1) [B, f*h*w, dim], e ~N(0,0.1) [B, 6, dim], context ~N(0,1)."""
    g = torch.Generator().manual_seed(seed)
    n = grid[0] * grid[1] * grid[2]
    x = torch.randn(batch, n, cfg.dim, generator=g).to(x_dtype)
    e = 0.1 * torch.randn(batch, 6, cfg.dim, generator=g)
    context = torch.randn(batch, ctx_len, cfg.dim, generator=g)
    seq_lens = torch.full((batch,), n, dtype=torch.long)
    grid_sizes = torch.tensor([list(grid)] * batch, dtype=torch.long)
    context_lens = torch.full((batch,), ctx_len, dtype=torch.long)
    return {
        "x": x.to(device),
        "e": e.to(device),
        "seq_lens": seq_lens,
        "grid_sizes": grid_sizes,
        "context": context.to(device),
        "context_lens": context_lens,
    }


def model_inputs(cfg: WanConfig, latent_fhw: tuple[int, int, int], batch: int, seed: int, t: float = 500.0,
                 device="cpu"):
    """Config 3/4 inputs: latent ~N(0,1) [16, F, H, W] and text context ~N(0,1) [512, 4096] per
    sample; CFG batch 2 = two samples with the same timestep."""
    g = torch.Generator().manual_seed(seed)
    f, h, w = latent_fhw
    xs = [torch.randn(cfg.in_dim, f, h, w, generator=g).to(device) for _ in range(batch)]
    ctx = [torch.randn(cfg.text_len, cfg.text_dim, generator=g).to(device) for _ in range(batch)]
    seq_len = f * (h // cfg.patch[1]) * (w // cfg.patch[2])
    return {"x": xs, "t": torch.full((batch,), float(t)), "context": ctx, "seq_len": seq_len}


def stock_bf16_model(cfg: WanConfig, state: dict, device, num_layers: int | None = None) -> "WanModelRef":
    """The stock forward in bf16 mixed precision with the weights of `state`: Linear and
    attention in bf16; time embedding, time projection and the modulation vectors fp32 (the
    reference's "eager" baseline, coda_wan/run_wan_coda.py:248-252)."""
    m = model_on_device(cfg, torch.bfloat16, device, seed=0, num_layers=num_layers)
    m.load_state_dict(state, strict=True)
    freqs, m.freqs = m.freqs, None
    m = m.to(torch.bfloat16)
    m.freqs = freqs
    m.time_embedding.float()
    m.time_projection.float()
    for b in m.blocks:
        b.modulation.data = b.modulation.data.float()
    m.head.modulation.data = m.head.modulation.data.float()
    return m.eval()
