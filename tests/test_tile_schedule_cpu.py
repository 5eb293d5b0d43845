"""Tile schedules of csrc/gemm.cu restated in Python. The one-launch norm GEMM (kEpiNorm):
every (row block, N tile) is visited exactly once; each CTA (pair) takes (row group, normalized
group) units u = c, c + CTAs, ..., each being the group's N tiles in order followed by the
group's even share of that row group's plain tiles (a remainder rotating over the groups with
the row group); when the plain tiles split evenly (all Wan shapes) the busiest CTA gets at
most one unit more than the average. The GPU test test_gemm_norm_fused_equals_split checks the kernel's output on
the same shapes; this checks the arithmetic for many more grids."""
import itertools

import pytest


def schedule(m_blocks, n_blocks, norm_groups, unit_tiles, pair, grid):
    """Mirror of the kernel's per-CTA sequence (gemm.cu, `coords` for kEpiNorm): a list of
    (row group, N tile, position inside the unit or -1) per CTA (pair)."""
    mg = (m_blocks + 1) // 2 if pair else m_blocks
    units = mg * norm_groups
    plain = n_blocks - norm_groups * unit_tiles
    vbase, vrem = divmod(plain, norm_groups)
    G = grid // 2 if pair else grid
    out = {}
    for c in range(G):
        seq = []
        for u in range(c, units, G):
            mq, g = divmod(u, norm_groups)
            seq += [(mq, g * unit_tiles + k, k) for k in range(unit_tiles)]

            def count(g2):
                return vbase + (1 if (g2 + mq) % norm_groups < vrem else 0)

            v0 = norm_groups * unit_tiles + sum(count(g2) for g2 in range(g))
            seq += [(mq, v0 + k, -1) for k in range(count(g))]
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
    flat = [t[:2] for s in seqs.values() for t in s]
    assert sorted(flat) == sorted(itertools.product(range(mg), range(n_blocks)))
    for s in seqs.values():
        # a unit: the group's tiles of one row group in order, then plain tiles of the same row group
        k = 0
        while k < len(s):
            assert s[k][2] == 0
            unit = s[k:k + tpu]
            assert [t[2] for t in unit] == list(range(tpu)) and len({t[0] for t in unit}) == 1
            assert [t[1] for t in unit] == list(range(unit[0][1], unit[0][1] + tpu))
            k += tpu
            while k < len(s) and s[k][2] == -1:
                assert s[k][0] == unit[0][0] and s[k][1] >= groups * tpu
                k += 1
    loads = [len(s) for s in seqs.values()]
    per_unit = tpu + -(-(n_blocks - groups * tpu) // groups)
    if (n_blocks - groups * tpu) % groups == 0:  # every unit equally long (all Wan shapes)
        assert max(loads) <= -(-len(flat) // len(loads)) + per_unit


def test_tail_of_the_cfg3_qkv_schedule():
    """cfg3 QKV on 74 CTA pairs: at most 63 tiles per pair against 62.3 on average."""
    seqs, _ = schedule(512, 18, 2, 6, True, 148)
    assert max(len(s) for s in seqs.values()) == 63


def raster(t, mg, n_blocks, group=8):
    """Mirror of gemm.cu's tile_coords: tile t -> (row block, N block), groups of `group` row
    blocks, row-minor inside a group (group 1: row-major)."""
    per = group * n_blocks
    grp = t // per
    first = grp * group
    gm = min(group, mg - first)
    r = t - grp * per
    n = r // gm
    return first + (r - n * gm), n


@pytest.mark.parametrize("group", [1, 8])
@pytest.mark.parametrize("mg", [1, 2, 7, 8, 9, 17, 32, 256, 591])
@pytest.mark.parametrize("n_blocks", [1, 6, 18, 35, 54, 60])
def test_grouped_rasterization_is_a_permutation(mg, n_blocks, group):
    tiles = [raster(t, mg, n_blocks, group) for t in range(mg * n_blocks)]
    assert sorted(tiles) == sorted(itertools.product(range(mg), range(n_blocks)))
    if group == 1:
        assert tiles == [divmod(t, n_blocks) for t in range(mg * n_blocks)]  # row-major


def test_grouped_rasterization_bounds_the_tiles_in_flight():
    """74 CTA pairs working on consecutive tiles of the 14B FFN1 at M = 151200 (591 pair row
    blocks x 54 N blocks) touch at most 8 row blocks and 10 N blocks at a time, so the weight
    columns in flight (10 x 2.6 MB) and the A rows (8 x 2.6 MB) fit in L2 together."""
    mg, nb = 591, 54
    for start in range(0, mg * nb - 74, 997):
        window = [raster(t, mg, nb) for t in range(start, start + 74)]
        assert len({m for m, _ in window}) <= 16 and len({n for _, n in window}) <= 11


def test_exchange_v_staging_layout():
    """The exchange GEMM's v staging (gemm.cu, kEpiNorm with peer stores): lane l (row l of the
    warp's 32) writes its 16-byte piece p (0-7: two 32-column chunks) at l*128 + ((p ^ (l & 7))
    << 4) of the warp's 4 KB; store step i has lane l read row 4i + l/8, piece l % 8. Every read
    gets the piece its (row, piece) names, each step covers 4 whole 128-byte rows (one line per
    8 lanes), and every quarter-warp's 8 accesses hit 8 distinct 16-byte bank groups (no shared
    memory bank conflict)."""
    def addr(row, piece):
        return row * 128 + ((piece ^ (row & 7)) << 4)

    written = {}
    for piece in range(8):
        addrs = [addr(lane, piece) for lane in range(32)]
        for q in range(4):  # quarter-warps
            assert len({(a % 128) // 16 for a in addrs[8 * q:8 * q + 8]}) == 8
        for lane, a in enumerate(addrs):
            assert a not in written
            written[a] = (lane, piece)
    assert sorted(written) == list(range(0, 4096, 16))
    for i in range(8):
        got = []
        for lane in range(32):
            row, piece = 4 * i + (lane >> 3), lane & 7
            a = addr(row, piece)
            assert written[a] == (row, piece)
            got.append((row, piece))
        for q in range(4):
            assert len({(addr(*rp) % 128) // 16 for rp in got[8 * q:8 * q + 8]}) == 8
            assert {rp[0] for rp in got[8 * q:8 * q + 8]} == {4 * i + q}  # one whole row per 8 lanes
