"""The sampling loop (CFG batch-2 forward + guidance combine + UniPC) driving the fused model
vs the same loop driving the fp32 stock-Wan oracle model, on the GPU: final latents after 3
steps within the multi-layer tolerance (relative L2 <= 2e-2)."""
import pytest
import torch

from oracle import wan_ref

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("solver", ["unipc", "euler"])
def test_sampler_with_fused_model_matches_oracle(pkg, solver):
    cfg = wan_ref.WAN_1_3B
    ref = wan_ref.init_weights_(wan_ref.WanModelRef(cfg, torch.float32, num_layers=2), seed=51).to(DEV)
    params = pkg.build_wan(pkg.WAN_1_3B, seed=0, device=DEV, num_layers=2)
    params.load_state_dict(ref.state_dict(), strict=True)
    params.to(torch.bfloat16)
    params.time_embedding.float()
    params.time_projection.float()
    for b in params.blocks:
        b.modulation.data = b.modulation.data.float()
    params.head.modulation.data = params.head.modulation.data.float()
    fused = pkg.FusedWanModel(params)
    inp = wan_ref.model_inputs(cfg, (2, 16, 24), 1, seed=52, device=DEV)
    g = torch.Generator(device="cpu").manual_seed(53)
    null = [0.1 * torch.randn(c.shape, generator=g).to(DEV, c.dtype) for c in inp["context"]]
    kw = dict(steps=3, guide_scale=5.0, shift=5.0, solver=solver)
    got = pkg.sampler.sample(fused, inp["x"], inp["context"], null, inp["seq_len"], **kw)
    with torch.no_grad():
        want = pkg.sampler.sample(ref, inp["x"], inp["context"], null, inp["seq_len"], input_dtype=torch.float32,
                                  **kw)
    pkg._lib.raise_on_device_error()
    for a, b in zip(got, want):
        assert a.shape == b.shape
        rel = ((a.float() - b.float()).norm() / b.float().norm()).item()
        assert rel <= 2e-2, rel
