"""The stream-K GEMM's division of work (gemm_i8_streamk.cuh, SkRun), restated and checked on
the CPU for the shapes the library may send it: every (tile, k-block) unit is computed once;
a tile is cut at most once; a cut tile is a STORE at the start of CTA c + 1 and a FINISH at
the end of CTA c (so a FINISH waits on a partial its neighbour writes first thing, and the
slots it reads stay inside the workspace)."""
import pytest


def runs(tiles, num_kb, G):
    """Segments (tile, kb0, kb1) of every CTA, as SkRun::next produces them."""
    total = tiles * num_kb
    out = []
    for c in range(G):
        u, end = total * c // G, total * (c + 1) // G
        segs = []
        while u < end:
            tile, kb0 = divmod(u, num_kb)
            kb1 = min(num_kb, kb0 + (end - u))
            segs.append((tile, kb0, kb1))
            u += kb1 - kb0
        out.append(segs)
    return out


SHAPES = [(152, 20, 148), (160, 32, 148), (160, 76, 148), (1536, 20, 148), (640, 76, 148), (2560, 32, 148),
          (148, 20, 148), (149, 1, 148), (300, 3, 148), (19456, 20, 148), (5, 7, 5), (9, 2, 8)]


@pytest.mark.parametrize('tiles,num_kb,G', SHAPES)
def test_units_once_and_cut_tiles_pair_up(tiles, num_kb, G):
    assert tiles >= G
    segs = runs(tiles, num_kb, G)
    covered = {}
    for c, ss in enumerate(segs):
        for i, (t, kb0, kb1) in enumerate(ss):
            assert 0 <= kb0 < kb1 <= num_kb
            for kb in range(kb0, kb1):
                assert (t, kb) not in covered
                covered[t, kb] = c
            if kb0 > 0:                                  # STORE: first segment, runs to the tile's end
                assert i == 0 and kb1 == num_kb and c > 0
                prev = segs[c - 1][-1]
                assert prev == (t, 0, kb0)               # CTA c - 1 finishes it
            elif kb1 < num_kb:                           # FINISH: last segment
                assert i == len(ss) - 1 and c + 1 < G   # reads slot c + 1 < G
                assert segs[c + 1][0] == (t, kb1, num_kb)
    assert len(covered) == tiles * num_kb
    # each tile in at most two CTAs
    owners = {}
    for (t, _), c in covered.items():
        owners.setdefault(t, set()).add(c)
    assert max(len(v) for v in owners.values()) <= 2


def test_critical_path_is_the_even_share():
    """Config 0 (M 512, N 9728 at 128 x 256: 152 tiles, 20 k-blocks) on 148 SMs: the
    data-parallel grid's longest CTA runs 2 tiles = 40 k-blocks; stream-K's runs 21."""
    segs = runs(152, 20, 148)
    longest = max(sum(kb1 - kb0 for _, kb0, kb1 in ss) for ss in segs)
    assert longest == 21
