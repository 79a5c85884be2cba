"""The decode-kernel timeline summariser (sqb200.timeline) on a synthetic file laid
out as the library writes it (no GPU)."""
import numpy as np

from sqb200 import timeline as TL


def write_fake(path, G=2, L=1, with_tiles=True):
    S = 8 * (5 * L + 1) + 6
    tl = np.zeros((G, S), np.uint64)
    for c in range(G):
        clk = 1000 + 10 * c
        tl[c, 0] = clk
        for s in range(5 * L + 1):
            for k in (1, 3, 2, 4, 5, 6):
                clk += 100
                tl[c, 8 * s + k] = clk
        tl[c, S - 2] = clk + 100
        tl[c, S - 1] = clk + 200
        # (global ns, clock) pairs at start and end: 1 ns a clock
        tl[c, S - 6], tl[c, S - 5] = 5000 + 1000 + 10 * c, 1000 + 10 * c
        tl[c, S - 4], tl[c, S - 3] = 5000 + clk + 200, clk + 200
    with open(path, "wb") as f:
        f.write(np.array([G, S], np.int32).tobytes())
        f.write(tl.tobytes())
        if with_tiles:
            mt = 2
            f.write(np.array([mt], np.int32).tobytes())
            tt = np.zeros((G, mt, 3), np.uint64)
            tb = np.zeros((G, mt, 2), np.int32)
            for c in range(G):
                for j in range(mt):
                    tt[c, j] = (1100 + 50 * j, 1300 + 50 * j, 1500 + 50 * j)
                    tb[c, j] = (16 * j, (0 << 16) | (j << 12) | 16)  # layer 0, kinds qkv / o, 16 rows
            f.write(tt.tobytes())
            f.write(tb.tobytes())


def test_summary_reads_the_library_layout(tmp_path):
    p = str(tmp_path / "tl.bin")
    write_fake(p)
    out = TL.summarise(p)
    assert "CTAs 2, layers 1" in out
    for kind in ("qkv", "attn", "o", "gu", "down", "lm"):
        assert any(line.startswith(kind) for line in out.splitlines()), kind
    tiles = [l for l in out.splitlines() if l.startswith("qkv ") or l.startswith("o ")]
    assert len(tiles) >= 2  # one stage row and one tile row each
    # tile 0: issued at 1100, consumer start at 1300 (1 ns a clock) -> 0.20 us
    assert any("0.20" in l for l in tiles)


def test_summary_without_tile_stamps(tmp_path):
    p = str(tmp_path / "tl.bin")
    write_fake(p, with_tiles=False)
    out = TL.summarise(p)
    assert "tiles" not in out
