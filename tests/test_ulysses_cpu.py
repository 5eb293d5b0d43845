"""Token-sharded self-attention regrouping on CPU ranks (gloo, world size 2 and 4): the layout
maps of oracle/ulysses_ref.py around a real all_to_all reproduce full-sequence attention.
Also: the unit assignment covers every (batch, head) pair once, including 12 heads x CFG
batch 2 on 8 ranks."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F

from oracle import ulysses_ref


@pytest.mark.parametrize("B,H,P", [(2, 12, 8), (1, 12, 4), (2, 12, 2), (2, 40, 8), (1, 40, 8)])
def test_unit_assignment_is_a_partition(B, H, P):
    U, owner = ulysses_ref.units(B, H, P)
    flat = [bh for d in owner for bh in d]
    assert len(flat) == B * H == len(set(flat)) and U * P == B * H


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, B, L, H, hd, q, k, v, ret):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        Lp = L // world
        D = H * hd
        rows = torch.cat([t[:, rank * Lp:(rank + 1) * Lp].reshape(B * Lp, D) for t in (q, k, v)], dim=1)
        U = B * H // world
        send = ulysses_ref.pack(rows, B, Lp, H, hd, 3, world)
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send)
        full = ulysses_ref.seq_gather(recv, 3, U, world, Lp, hd)
        o = F.scaled_dot_product_attention(full[0][None], full[1][None], full[2][None])[0]
        send2 = ulysses_ref.seq_scatter(o, U, world, Lp, hd)
        recv2 = torch.empty_like(send2)
        dist.all_to_all_single(recv2, send2)
        y = ulysses_ref.unpack(recv2, B, Lp, H, hd, world)
        ret[rank] = y
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,B,H", [(2, 2, 12), (4, 2, 12)])
def test_regroup_equals_full_attention(world, B, H):
    torch.manual_seed(0)
    L, hd = 8 * world, 16
    q, k, v = (torch.randn(B, L, H * hd) for _ in range(3))
    mgr = mp.Manager()
    ret = mgr.dict()
    mp.start_processes(_worker, args=(world, _free_port(), B, L, H, hd, q, k, v, ret), nprocs=world,
                       start_method="spawn", join=True)
    Lp = L // world
    ref = F.scaled_dot_product_attention(
        q.view(B, L, H, hd).transpose(1, 2), k.view(B, L, H, hd).transpose(1, 2), v.view(B, L, H, hd).transpose(1, 2)
    ).transpose(1, 2).reshape(B, L, H * hd)
    for r in range(world):
        want = ref[:, r * Lp:(r + 1) * Lp].reshape(B * Lp, H * hd)
        assert torch.allclose(ret[r], want, atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("B,Lp,H,P", [(2, 16380, 12, 2), (2, 4095, 12, 8), (2, 8190, 40, 4), (1, 7, 12, 3)])
def test_p2p_exchange_layout(pkg, B, Lp, H, P):
    """The NVLink exchange region: 256-byte aligned, disjoint parts that hold exactly the
    q/k/v of this rank's units for all tokens (twice) and the attention rows of its tokens."""
    if (B * H) % P:
        pytest.skip("units do not divide")
    hd = 128
    lay = pkg.ulysses.exchange_layout(B, Lp, H, hd, P)
    U, L = B * H // P, P * Lp
    assert lay["full_bytes"] == 3 * U * L * hd * 2 and lay["y_bytes"] == B * Lp * H * hd * 2
    parts = [(o, lay["full_bytes"]) for o in lay["full_off"]] + [(o, lay["y_bytes"]) for o in lay["y_off"]] + \
        [(o, 4 * P) for o in lay["flag_off"]]
    for o, n in parts:
        assert o % 256 == 0 and o + n <= lay["total"]
    spans = sorted(parts)
    for (o1, n1), (o2, _) in zip(spans, spans[1:]):
        assert o1 + n1 <= o2


def _padded_worker(rank, world, port, B, L, H, hd, lens, q, k, v, ret):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from __graft_entry__ import load_package

        sp = load_package().SeqParallel(None, world, rank, (1, 1, L), L, transport="nccl")
        Lp = L // world
        D = H * hd
        rows = torch.cat([t[:, rank * Lp:(rank + 1) * Lp].reshape(B * Lp, D) for t in (q, k, v)], dim=1)
        U = B * H // world
        send = ulysses_ref.pack(rows, B, Lp, H, hd, 3, world)
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send)
        full = ulysses_ref.seq_gather(recv, 3, U, world, Lp, hd)
        mask = sp.unit_key_mask(lens, B, H, L, "cpu")
        o = F.scaled_dot_product_attention(full[0][None], full[1][None], full[2][None], attn_mask=mask)[0]
        send2 = ulysses_ref.seq_scatter(o, U, world, Lp, hd)
        recv2 = torch.empty_like(send2)
        dist.all_to_all_single(recv2, send2)
        ret[rank] = ulysses_ref.unpack(recv2, B, Lp, H, hd, world)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,B,H,lens", [(2, 2, 12, [16, 11]), (4, 2, 12, [5, 32])])
def test_regroup_masks_padded_keys(world, B, H, lens):
    """Token-sharded attention with a sample shorter than the padded length: each rank masks its
    units' keys past their sample's length (SeqParallel.unit_key_mask), which equals the
    single-GPU path's per-sample key mask."""
    torch.manual_seed(1)
    L, hd = 8 * world, 16
    q, k, v = (torch.randn(B, L, H * hd) for _ in range(3))
    mgr = mp.Manager()
    ret = mgr.dict()
    mp.start_processes(_padded_worker, args=(world, _free_port(), B, L, H, hd, lens, q, k, v, ret), nprocs=world,
                       start_method="spawn", join=True)
    Lp = L // world
    kl = torch.tensor(lens).view(B, 1, 1, 1)
    mask = torch.arange(L).view(1, 1, 1, L) < kl
    ref = F.scaled_dot_product_attention(
        q.view(B, L, H, hd).transpose(1, 2), k.view(B, L, H, hd).transpose(1, 2), v.view(B, L, H, hd).transpose(1, 2),
        attn_mask=mask).transpose(1, 2).reshape(B, L, H * hd)
    unmasked = F.scaled_dot_product_attention(
        q.view(B, L, H, hd).transpose(1, 2), k.view(B, L, H, hd).transpose(1, 2),
        v.view(B, L, H, hd).transpose(1, 2)).transpose(1, 2).reshape(B, L, H * hd)
    assert not torch.allclose(ref, unmasked, atol=1e-3)  # the padding matters for this case
    for r in range(world):
        want = ref[:, r * Lp:(r + 1) * Lp].reshape(B * Lp, H * hd)
        assert torch.allclose(ret[r], want, atol=1e-5, rtol=1e-5)


def test_unit_key_mask_none_without_padding(pkg):
    sp = pkg.SeqParallel(None, 8, 3, (1, 1, 64), 64, transport="nccl")
    assert sp.unit_key_mask(None, 2, 12, 64, "cpu") is None
    assert sp.unit_key_mask([64, 64], 2, 12, 64, "cpu") is None
    m = sp.unit_key_mask([64, 40], 2, 12, 64, "cpu")
    # rank 3 of 8 holds units 9, 10, 11 (batch 0, heads 9-11): nothing masked
    assert m.shape == (1, 3, 1, 64) and bool(m.all())
    m = pkg.SeqParallel(None, 8, 5, (1, 1, 64), 64, transport="nccl").unit_key_mask([64, 40], 2, 12, 64, "cpu")
    # rank 5 holds units 15, 16, 17 (batch 1): keys 40.. masked
    assert bool(m[..., :40].all()) and not bool(m[..., 40:].any())


def _direct_store_offsets(rank, B, Lp, H, P, mat):
    """The peer-store address rule of the exchanging kernels (xchg_addr in csrc/gemm.cu and the
    same rule in csrc/p2p.cu), restated: element (row, column c) of matrix `mat` of rank
    `rank`'s QKV output goes to rank pr's region, element offset ((mat*U + ul)*L + gtok)*128 +
    c % 128, with unit u = b*H + c // 128, pr = u // U, ul = u % U, gtok = rank*Lp + token."""
    U, L, D = B * H // P, P * Lp, H * 128
    row = torch.arange(B * Lp).view(-1, 1)
    c = torch.arange(D).view(1, -1)
    b = row // Lp
    u = b * H + (c >> 7)
    pr = u // U
    ul = u - pr * U
    gtok = rank * Lp + (row - b * Lp)
    return pr, ((mat * U + ul) * L + gtok) * 128 + (c & 127)


@pytest.mark.parametrize("B,H,P,Lp", [(2, 12, 2, 5), (2, 12, 4, 3), (2, 12, 8, 2), (1, 12, 4, 3), (2, 40, 8, 2)])
def test_direct_peer_stores_land_where_the_gather_puts_them(B, H, P, Lp):
    """Stores made with the address rule cover every slot of every rank's q/k/v region exactly
    once and leave there what pack -> all_to_all -> seq_gather (the layout oracle) produces."""
    torch.manual_seed(1)
    U, L, D = B * H // P, P * Lp, H * 128
    rows = [torch.randn(B * Lp, 3 * D) for _ in range(P)]
    region = [torch.full((3 * U * L * 128,), float("nan")) for _ in range(P)]
    hits = [torch.zeros(3 * U * L * 128, dtype=torch.int64) for _ in range(P)]
    for r in range(P):
        for mat in range(3):
            pr, off = _direct_store_offsets(r, B, Lp, H, P, mat)
            vals = rows[r][:, mat * D:(mat + 1) * D]
            for d in range(P):
                sel = pr == d
                region[d][off[sel]] = vals[sel]
                hits[d].index_add_(0, off[sel], torch.ones_like(off[sel]))
    sends = [ulysses_ref.pack(rows[r], B, Lp, H, 128, 3, P) for r in range(P)]
    for d in range(P):
        assert torch.equal(hits[d], torch.ones_like(hits[d])), d
        recv = torch.stack([sends[p][d] for p in range(P)])  # what all_to_all delivers to rank d
        want = ulysses_ref.seq_gather(recv, 3, U, P, Lp, 128)
        assert torch.equal(region[d].view(3, U, L, 128), want), d
