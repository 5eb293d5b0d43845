"""Token-sharded (sequence-parallel) forward on 2 (and 4) GPUs: every rank's output shard equals
the same tokens of the single-GPU forward (same weights and inputs), for each Ulysses transport:
NVLink peer stores with the QKV GEMM storing into the peers itself (gemm_exchange), peer stores
by the separate exchange kernel, and the NCCL all-to-all. Cases needing more GPUs than are
visible are skipped."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

LAYERS, LATENT = 3, (2, 16, 24)  # 2 x 8 x 12 = 192 tokens per sample


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _inputs(cfg, dev, padded=False):
    from oracle import wan_ref

    inp = wan_ref.model_inputs(cfg, LATENT, 2, seed=5, device=dev)
    if padded:
        # both samples' 192 tokens padded to a 256-token sequence (as stock Wan pads to its
        # fixed seq_len): the padding keys (on rank 1 of 2) must be masked on every rank
        inp["seq_len"] = 256
    return inp


def _worker(rank, world, port, root, transport, padded, gemm_exchange, ret):
    import sys
    from datetime import timedelta

    sys.path.insert(0, root)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=120))
    try:
        from __graft_entry__ import load_package
        from oracle import wan_ref

        pkg = load_package()
        cfg = wan_ref.WAN_1_3B
        inp = _inputs(cfg, dev, padded)
        L = inp["seq_len"]
        sp = pkg.SeqParallel(dist.group.WORLD, world, rank, (LATENT[0], LATENT[1] // 2, LATENT[2] // 2), L,
                             transport=transport, gemm_exchange=gemm_exchange)
        params = pkg.build_wan(pkg.WAN_1_3B, seed=11, device=dev, num_layers=LAYERS)
        model = pkg.FusedWanModel(params, sp)
        with torch.no_grad():
            y = model(inp["x"], inp["t"], inp["context"], L)
            y2 = model(inp["x"], inp["t"], inp["context"], L)  # second forward: the other exchange buffers
        torch.cuda.synchronize()
        pkg._lib.raise_on_device_error()
        ret[rank] = (y.float().cpu(), y2.float().cpu())
        sp.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,transport,padded,gemm_exchange", [
    (2, "p2p", False, True), (2, "p2p", False, False), (2, "nccl", False, False),
    (2, "p2p", True, True), (2, "p2p", True, False), (2, "nccl", True, False),
    (4, "p2p", False, True), (4, "p2p", False, False), (4, "p2p", True, True),
])
def test_sequence_parallel_matches_single_gpu(pkg, world, transport, padded, gemm_exchange):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from pathlib import Path

    from oracle import wan_ref

    root = str(Path(__file__).resolve().parents[1])
    dev = torch.device("cuda", 0)
    cfg = wan_ref.WAN_1_3B
    inp = _inputs(cfg, dev, padded)
    L = inp["seq_len"]
    params = pkg.build_wan(pkg.WAN_1_3B, seed=11, device=dev, num_layers=LAYERS)
    with torch.no_grad():
        full = pkg.FusedWanModel(params)(inp["x"], inp["t"], inp["context"], L, return_tokens=True).float().cpu()
    ret = mp.Manager().dict()
    mp.start_processes(_worker, args=(world, _port(), root, transport, padded, gemm_exchange, ret), nprocs=world,
                       start_method="spawn", join=True)
    Lp = L // world
    for r in range(world):
        want = full[:, r * Lp:(r + 1) * Lp]
        got, got2 = ret[r]
        rel = ((got - want).norm() / want.norm()).item()
        assert rel < 1e-2, (r, rel)
        assert torch.equal(got, got2), r  # deterministic across epochs / buffers
