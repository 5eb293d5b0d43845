"""The tile schedule of the one-launch norm GEMM (kEpiNorm in csrc/gemm.cu), restated in Python:
every (row block, N tile) is visited exactly once, each CTA (pair) gets whole (row block, group)
units first and then a contiguous range of the plain tiles, and no CTA gets more than
ceil(tiles / CTAs) + the unit remainder. The GPU test test_gemm_norm_fused_equals_split checks
the kernel's output on the same shapes; this checks the arithmetic for many more grids."""
import itertools

import pytest


def schedule(m_blocks, n_blocks, norm_groups, unit_tiles, pair, grid):
    """Mirror of the kernel's per-CTA sequence (gemm.cu, `coords` for kEpiNorm)."""
    mg = (m_blocks + 1) // 2 if pair else m_blocks
    units = mg * norm_groups
    plain = n_blocks - norm_groups * unit_tiles
    G = grid // 2 if pair else grid
    out = {}
    for c in range(G):
        base, rem = units // G, units % G
        su = base + (1 if c < rem else 0)
        P = mg * plain
        T = (units * unit_tiles + P + G - 1) // G
        v1 = max(0, T - unit_tiles * (base + 1))
        v0 = max(0, T - unit_tiles * base)
        vs = min(c, rem) * v1 + max(0, c - rem) * v0
        ve = min(vs + (v1 if c < rem else v0), P)
        vs = min(vs, P)
        seq = []
        for i in range(su * unit_tiles + (ve - vs)):
            nu = su * unit_tiles
            if i < nu:
                j, up = divmod(i, unit_tiles)
                u = c + j * G
                mq = u // norm_groups
                nb = (u - mq * norm_groups) * unit_tiles + up
            else:
                pidx = vs + (i - nu)
                mq, nb = divmod(pidx, plain)
                nb += norm_groups * unit_tiles
            seq.append((mq, nb))
        out[c] = seq
    return out, mg


@pytest.mark.parametrize("M", [1, 128, 129, 300, 4095, 8190, 16380, 65520, 151200])
@pytest.mark.parametrize("N,groups,width", [(4608, 2, 1536), (1536, 1, 1536), (3072, 1, 1536),
                                            (15360, 2, 5120), (512, 2, 256), (576, 2, 256)])
@pytest.mark.parametrize("pair,grid", [(False, 148), (True, 148), (True, 10), (False, 7)])
def test_every_tile_once_and_units_whole(M, N, groups, width, pair, grid):
    if pair and M <= 256:
        pytest.skip("pairs run only above 256 rows")
    m_blocks, n_blocks = (M + 127) // 128, (N + 255) // 256
    tpu = width // 256
    seqs, mg = schedule(m_blocks, n_blocks, groups, tpu, pair, grid)
    flat = [t for s in seqs.values() for t in s]
    assert sorted(flat) == sorted(itertools.product(range(mg), range(n_blocks)))
    for s in seqs.values():
        # units first: each normalized group's tiles of one row block come consecutively, in order
        k = 0
        while k < len(s) and s[k][1] < groups * tpu:
            unit = s[k:k + tpu]
            assert [t[1] for t in unit] == list(range(unit[0][1], unit[0][1] + tpu))
            assert unit[0][1] % tpu == 0 and len({t[0] for t in unit}) == 1
            k += tpu
        assert all(t[1] >= groups * tpu for t in s[k:])  # then plain tiles only


def test_tail_of_the_cfg3_qkv_schedule():
    """cfg3 QKV on 74 CTA pairs: at most 63 tiles per pair against 62.3 on average."""
    seqs, _ = schedule(512, 18, 2, 6, True, 148)
    assert max(len(s) for s in seqs.values()) == 63
