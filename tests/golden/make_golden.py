"""Generate tests/golden/*.npz from the reference's own code (run in the build container).

    WDIT_REFERENCE_DIR=<checkout of Owen718/CODA-Wan-DiT> TRITON_INTERPRET=1 python tests/golden/make_golden.py

Sources (Owen718/CODA-Wan-DiT, imported through oracle/reference_kernels.py):
  ln_mod.npz      _layernorm_modulation_kernel via layernorm_modulation_bf16 (wan_coda_kernels.py:35-81)
  rmsnorm.npz     _rmsnorm_kernel via rmsnorm_fused (:371-411)
  qk_rms_rope.npz _qk_rms_rope_kernel via qk_rms_rope_from_partials (:233-352)
  rope_table.npz  build_wan_rope_table (:414-430) for grid (2, 3, 4) plus the byte count of
                  the production table (21, 30, 52) (published: 16,773,120 bytes,
                  docs/report.md:150)
  prepack.npz     prepack_linear_inplace / prepack_qk_inplace (:433-461) on a small Linear

bf16 tensors are stored as their uint16 bit patterns. Inputs are seeded (seed per file).
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"
ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402

from oracle import reference_kernels  # noqa: E402
from oracle.wan_ref import rope_freqs  # noqa: E402

OUT = Path(__file__).resolve().parent
DIM = 1536


def bits(t: torch.Tensor) -> np.ndarray:
    assert t.dtype == torch.bfloat16
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def main() -> None:
    R = reference_kernels.load()
    g = torch.Generator().manual_seed(1234)

    # LayerNorm + modulation: fp32 rows (with an offset-mean row), and bf16 rows.
    rows = 6
    x = torch.randn(rows, DIM, generator=g)
    x[1] += 5.0  # offset mean
    x[2] *= 30.0  # large variance
    scale = 0.1 * torch.randn(DIM, generator=g)
    shift = 0.1 * torch.randn(DIM, generator=g)
    out = R.layernorm_modulation_bf16(x, scale, shift, 1e-6)
    xb = torch.randn(rows, DIM, generator=g).to(torch.bfloat16)
    outb = R.layernorm_modulation_bf16(xb, scale, shift, 1e-6)
    np.savez(OUT / "ln_mod.npz", x=x.numpy(), scale=scale.numpy(), shift=shift.numpy(), out=bits(out),
             xb=bits(xb), outb=bits(outb), eps=np.float32(1e-6))

    # Full-width RMSNorm of bf16 rows.
    xr = (2.0 * torch.randn(rows, DIM, generator=g)).to(torch.bfloat16)
    w = (1.0 + 0.1 * torch.randn(DIM, generator=g)).to(torch.bfloat16)
    outr = R.rmsnorm_fused(xr, w, 1e-6)
    np.savez(OUT / "rmsnorm.npz", x=bits(xr), w=bits(w), out=bits(outr), eps=np.float32(1e-6))

    # q/k RMSNorm + RoPE from mean-square partials (in place over a [rows, 3072] buffer).
    qk = torch.randn(rows, 2 * DIM, generator=g).to(torch.bfloat16)
    partial = qk.float().square().view(rows, 24, 128).mean(-1)
    wq = (1.0 + 0.1 * torch.randn(DIM, generator=g)).to(torch.bfloat16)
    wk = (1.0 + 0.1 * torch.randn(DIM, generator=g)).to(torch.bfloat16)
    freqs = rope_freqs(1024, 128)
    cos_t, sin_t = R.build_wan_rope_table((1, 2, 3), freqs)
    cos_rows, sin_rows = cos_t[:rows].contiguous(), sin_t[:rows].contiguous()
    qk_in = qk.clone()
    q, k = R.qk_rms_rope_from_partials(qk.clone(), partial, wq, wk, cos_rows, sin_rows, 1e-6)
    np.savez(OUT / "qk_rms_rope.npz", qk=bits(qk_in), partial=partial.numpy(), wq=bits(wq), wk=bits(wk),
             cos=cos_rows.numpy(), sin=sin_rows.numpy(), q=bits(q.contiguous()), k=bits(k.contiguous()),
             eps=np.float32(1e-6))

    # RoPE table on a small grid + production byte count.
    cs, sn = R.build_wan_rope_table((2, 3, 4), freqs)
    cbig, sbig = R.build_wan_rope_table((21, 30, 52), freqs)
    nbytes = cbig.untyped_storage().nbytes() + sbig.untyped_storage().nbytes()
    np.savez(OUT / "rope_table.npz", cos=cs.numpy(), sin=sn.numpy(), grid=np.array([2, 3, 4]),
             prod_bytes=np.int64(nbytes), freqs_re=freqs.real.numpy()[:8], freqs_im=freqs.imag.numpy()[:8])

    # Prepack aliasing (small Linear).
    lin = torch.nn.Linear(64, 32)
    lq = torch.nn.Linear(64, 64)
    lk = torch.nn.Linear(64, 64)
    w0 = lin.weight.detach().clone()
    packed = R.prepack_linear_inplace(lin)
    qk_w, qk_b = R.prepack_qk_inplace(lq, lk)
    np.savez(OUT / "prepack.npz", w=w0.numpy(), packed=packed.numpy(), packed_shape=np.array(packed.shape),
             packed_contig=np.bool_(packed.is_contiguous()),
             alias=np.bool_(lin.weight.untyped_storage().data_ptr() == packed.untyped_storage().data_ptr()),
             qk_shape=np.array(qk_w.shape), qk_bias_shape=np.array(qk_b.shape))
    print("golden fixtures written to", OUT, "; production RoPE table bytes:", nbytes)


if __name__ == "__main__":
    main()
