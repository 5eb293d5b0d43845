"""Oracle pinned against the reference's own outputs (tests/golden, made by
tests/golden/make_golden.py from coda_wan/wan_coda_kernels.py) and its published known
answers. CPU only."""
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import fused_ref, wan_ref

GOLD = Path(__file__).resolve().parent / "golden"


def bf16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(a.astype(np.uint16).view(np.int16).copy()).view(torch.bfloat16)


def ulp_close(got: torch.Tensor, want: torch.Tensor, max_ulps: int = 1, min_exact: float = 0.99):
    """bf16 tensors equal up to `max_ulps` units in the last place, mostly bit-exact
    (reduction order may move a rounding boundary)."""
    def ordered(t):  # sign-magnitude bf16 bits -> monotone integers
        x = t.contiguous().view(torch.int16).to(torch.int32)
        return torch.where(x < 0, -(x & 0x7FFF), x)

    d = (ordered(got) - ordered(want)).abs()
    assert int(d.max()) <= max_ulps, f"max ulp diff {int(d.max())}"
    assert float((d == 0).float().mean()) >= min_exact


# The fixtures come from Triton's CPU interpreter, which rounds fp32 -> bf16 toward zero
# (GPU Triton and CUDA round to nearest even). Matching them in "rz" mode pins the fp32
# arithmetic of each op; "rne" stays within one bf16 ulp of them.


def test_layernorm_modulation_matches_reference_kernel():
    z = np.load(GOLD / "ln_mod.npz")
    x, s, sh = (torch.from_numpy(z[k]) for k in ("x", "scale", "shift"))
    ulp_close(fused_ref.layernorm_modulation(x, s, sh, float(z["eps"]), mode="rz"), bf16(z["out"]))
    ulp_close(fused_ref.layernorm_modulation(bf16(z["xb"]), s, sh, float(z["eps"]), mode="rz"), bf16(z["outb"]))
    ulp_close(fused_ref.layernorm_modulation(x, s, sh, float(z["eps"])), bf16(z["out"]), min_exact=0.3)


def test_rmsnorm_matches_reference_kernel():
    z = np.load(GOLD / "rmsnorm.npz")
    ulp_close(fused_ref.rmsnorm(bf16(z["x"]), bf16(z["w"]), float(z["eps"]), mode="rz"), bf16(z["out"]))


def test_qk_rms_rope_matches_reference_kernel():
    z = np.load(GOLD / "qk_rms_rope.npz")
    q, k = fused_ref.qk_rms_rope_from_partials(
        bf16(z["qk"]), torch.from_numpy(z["partial"]), bf16(z["wq"]), bf16(z["wk"]), torch.from_numpy(z["cos"]),
        torch.from_numpy(z["sin"]), float(z["eps"]), mode="rz")
    # two intermediate roundings: allow the rare 2-ulp step where one moved a boundary
    ulp_close(q, bf16(z["q"]), max_ulps=2)
    ulp_close(k, bf16(z["k"]), max_ulps=2)


def test_rope_table_matches_reference_and_published_size():
    z = np.load(GOLD / "rope_table.npz")
    freqs = wan_ref.rope_freqs(1024, 128)
    assert np.allclose(freqs.real.numpy()[:8], z["freqs_re"]) and np.allclose(freqs.imag.numpy()[:8], z["freqs_im"])
    cos, sin = fused_ref.build_wan_rope_table(tuple(z["grid"]), freqs)
    assert torch.equal(cos, torch.from_numpy(z["cos"])) and torch.equal(sin, torch.from_numpy(z["sin"]))
    # Published storage delta of the shared table at grid (21, 30, 52): docs/report.md:150.
    assert int(z["prod_bytes"]) == 16_773_120 == 2 * 21 * 30 * 52 * 64 * 4
    # The complex table used by the block oracle agrees with the reference's cos/sin split.
    tab = wan_ref.rope_table(tuple(int(v) for v in z["grid"]), freqs)
    assert torch.equal(tab.real.float(), cos) and torch.equal(tab.imag.float(), sin)


def test_gelu_constants_known_answer():
    assert abs(fused_ref.GELU_C0 - (2.0 / np.pi) ** 0.5) < 1e-15
    assert fused_ref.GELU_C1 == 0.044715
    x = torch.linspace(-6, 6, 1001, dtype=torch.float64)
    assert torch.allclose(fused_ref.gelu_tanh(x), F.gelu(x, approximate="tanh"), atol=1e-12)


def test_prepack_semantics_of_reference():
    z = np.load(GOLD / "prepack.npz")
    # The reference transposes once into a contiguous (K, N) buffer that the parameter aliases.
    assert tuple(z["packed_shape"]) == (64, 32) and bool(z["packed_contig"]) and bool(z["alias"])
    assert np.array_equal(z["packed"], z["w"].T)
    assert tuple(z["qk_shape"]) == (64, 128) and tuple(z["qk_bias_shape"]) == (128,)


def test_partial_layout_and_merge_rule():
    # [M, 2*D/128] mean-square partials; rstd from the mean of the 12 partials of a half
    # equals the full-width RMS (wan_coda_kernels.py:204-206, 258-265).
    g = torch.Generator().manual_seed(3)
    a = torch.randn(5, 256, generator=g).to(torch.bfloat16)
    w = (0.02 * torch.randn(256, 3072, generator=g)).to(torch.bfloat16)
    qk, part = fused_ref.qk_linear_bias_partial_rms(a, w, torch.zeros(3072))
    assert part.shape == (5, 24)
    full = qk.float()[:, :1536].square().mean(-1)
    assert torch.allclose(part[:, :12].mean(-1), full, rtol=1e-6)


@pytest.mark.parametrize("offset", [0.0, 3.0, 20.0])
def test_ln_fold_algebra_exact(offset):
    """rstd*(x W' - mu colsum(W')) + shift^T W + b == (LN(x)(1+s) + shift) W + b, exactly in
    fp64; the fused kernels implement the left side."""
    g = torch.Generator().manual_seed(5)
    M, K, N = 7, 512, 96
    x = (torch.randn(M, K, generator=g) + offset).double()
    W = (0.02 * torch.randn(N, K, generator=g)).double()
    b = (0.01 * torch.randn(N, generator=g)).double()
    s = (0.1 * torch.randn(K, generator=g)).double()
    sh = (0.1 * torch.randn(K, generator=g)).double()
    mu = x.mean(-1, keepdim=True)
    rstd = torch.rsqrt(((x - mu) ** 2).mean(-1, keepdim=True) + 1e-6)
    want = (((x - mu) * rstd) * (1 + s) + sh) @ W.t() + b
    Wf = W * (1 + s)[None, :]
    got = rstd * (x @ Wf.t() - mu * Wf.sum(-1)[None, :]) + (W @ sh + b)[None, :]
    assert torch.allclose(got, want, rtol=1e-9, atol=1e-9)


def test_ln_stats_merge_matches_layernorm():
    g = torch.Generator().manual_seed(6)
    x = torch.randn(9, 1536, generator=g) * 3 + 7
    st = fused_ref.ln_stats(x)
    assert st.shape == (9, 6, 2)
    mu, rstd = fused_ref.merge_stats(st, 1536, 1e-6)
    assert torch.allclose(mu, x.mean(-1), rtol=1e-5, atol=1e-5)
    assert torch.allclose(rstd, torch.rsqrt(x.var(-1, unbiased=False) + 1e-6), rtol=1e-4)


def test_block_oracle_equals_op_chain():
    """The block oracle equals the chain of reference ops (fp32, tiny grid)."""
    cfg = wan_ref.WAN_1_3B
    torch.manual_seed(0)
    blk = wan_ref.init_weights_(wan_ref.WanBlockRef(cfg, torch.float32), seed=1, norm_jitter=0.1)
    grid = (1, 2, 4)
    inp = wan_ref.block_inputs(cfg, grid, 1, seed=2, ctx_len=16)
    freqs = wan_ref.rope_freqs(1024, 128)
    with torch.no_grad():
        out = blk(inp["x"].clone(), inp["e"], inp["seq_lens"], inp["grid_sizes"], freqs, inp["context"],
                  inp["context_lens"])
        x = inp["x"][0]
        e = (blk.modulation.float() + inp["e"].float())[0]
        L = x.shape[0]
        mu = x.mean(-1, keepdim=True)
        ln = (x - mu) * torch.rsqrt(((x - mu) ** 2).mean(-1, keepdim=True) + 1e-6)
        z = ln * (1 + e[1]) + e[0]
        sa = blk.self_attn
        q = z @ sa.q.weight.t() + sa.q.bias
        k = z @ sa.k.weight.t() + sa.k.bias
        v = z @ sa.v.weight.t() + sa.v.bias
        rms = lambda t, w: t * torch.rsqrt(t.square().mean(-1, keepdim=True) + 1e-6) * w
        q, k = rms(q, sa.norm_q.weight), rms(k, sa.norm_k.weight)
        cos, sin = fused_ref.build_wan_rope_table(grid, freqs)
        q, k = fused_ref.rope_rows(q, cos, sin), fused_ref.rope_rows(k, cos, sin)
        y = fused_ref.sdpa(q.view(1, L, 12, 128), k.view(1, L, 12, 128), v.view(1, L, 12, 128)).reshape(L, -1)
        x = x + (y @ sa.o.weight.t() + sa.o.bias) * e[2]
        n3 = blk.norm3
        mu = x.mean(-1, keepdim=True)
        c_in = (x - mu) * torch.rsqrt(((x - mu) ** 2).mean(-1, keepdim=True) + 1e-6) * n3.weight + n3.bias
        ca = blk.cross_attn
        cq = rms(c_in @ ca.q.weight.t() + ca.q.bias, ca.norm_q.weight)
        ctx = inp["context"][0]
        ck = rms(ctx @ ca.k.weight.t() + ca.k.bias, ca.norm_k.weight)
        cv = ctx @ ca.v.weight.t() + ca.v.bias
        cy = fused_ref.sdpa(cq.view(1, L, 12, 128), ck.view(1, -1, 12, 128), cv.view(1, -1, 12, 128)).reshape(L, -1)
        x = x + cy @ ca.o.weight.t() + ca.o.bias
        mu = x.mean(-1, keepdim=True)
        z = (x - mu) * torch.rsqrt(((x - mu) ** 2).mean(-1, keepdim=True) + 1e-6) * (1 + e[4]) + e[3]
        h = fused_ref.gelu_tanh(z @ blk.ffn[0].weight.t() + blk.ffn[0].bias)
        x = x + (h @ blk.ffn[2].weight.t() + blk.ffn[2].bias) * e[5]
    assert torch.allclose(out[0], x, rtol=1e-4, atol=1e-4)
