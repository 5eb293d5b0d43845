"""The product path has no CPU implementation: every op refuses host tensors loudly instead of
computing something (CPU only, no device needed)."""
import pytest
import torch

D = 1536


def _cases(ops):
    bf = lambda *s: torch.zeros(*s, dtype=torch.bfloat16)  # noqa: E731
    f32 = lambda *s: torch.zeros(*s, dtype=torch.float32)  # noqa: E731
    return {
        "gemm_act": lambda: ops.gemm_act(bf(64, 64), bf(64, 64)),
        "gemm_residual": lambda: ops.gemm_residual(bf(64, 64), bf(64, 64), f32(64, 64)),
        "gemm_norm": lambda: ops.gemm_norm(bf(64, 256), bf(256, 256), norm_groups=1, norm_width=128,
                                           norm_w=(f32(128), None)),
        "ln_stats": lambda: ops.ln_stats(f32(8, D)),
        "fold_weight": lambda: ops.fold_weight(bf(64, 64), mult_c=1.0),
        "fold_weight_batch": lambda: ops.fold_weight_batch([dict(w=bf(64, 64), mult_c=1.0)]),
        "patch_rows": lambda: ops.patch_rows(bf(16, 1, 4, 4), (1, 2, 2), 0, 4, 64),
        "cross_kv_layers": lambda: ops.cross_kv_layers(bf(8, 128), bf(2 * 256, 128), f32(512), f32(2, 128), 1e-6),
        "layernorm_modulation_bf16": lambda: ops.layernorm_modulation_bf16(f32(4, D), f32(D), f32(D), 1e-6),
        "linear_bias_gelu_fixed": lambda: ops.linear_bias_gelu_fixed(bf(4, D), bf(D, 64), f32(64)),
        "qk_rms_rope_from_partials": lambda: ops.qk_rms_rope_from_partials(
            bf(4, 2 * D), f32(4, 2 * D // 128), f32(D), f32(D), f32(4, 64), f32(4, 64), 1e-6),
        "rmsnorm_fused": lambda: ops.rmsnorm_fused(bf(4, D), f32(D), 1e-6),
        "linear_bias_residual_fixed": lambda: ops.linear_bias_residual_fixed(bf(4, D), bf(D, D), f32(4, D), f32(D)),
    }


NAMES = ["gemm_act", "gemm_residual", "gemm_norm", "ln_stats", "fold_weight", "fold_weight_batch", "patch_rows",
         "cross_kv_layers", "layernorm_modulation_bf16", "linear_bias_gelu_fixed", "qk_rms_rope_from_partials",
         "rmsnorm_fused", "linear_bias_residual_fixed"]


@pytest.mark.parametrize("name", NAMES)
def test_op_refuses_host_tensors(pkg, name):
    cases = _cases(pkg.ops)
    assert set(cases) == set(NAMES)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        cases[name]()
