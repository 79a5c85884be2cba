"""Summarise the persistent decode kernel's stage timeline.

With `SQ_DECODE_TIMELINE=<file>` set when a context is created, the library
records per-CTA stage timestamps of every decode launch and writes the last
launch's to <file> when the step is checked (int32 CTAs and stride, then
[CTAs][stride] u64 SM clocks with two (global ns, clock) pairs per CTA, then
int32 max_tiles, [CTAs][max_tiles][3] u64 tile clocks {issued, consumer start
(bytes landed and the consuming warp group there), released}
and the [CTAs][max_tiles] int2 tile table). Stages per layer: q/k/v, attention,
O, gate/up, down; the LM head last.

    python -m sqb200.timeline <file>

prints, per stage kind, the mean span from the previous stage's last CTA to this
stage's last CTA (the critical path), when the median CTA had its input in
registers and finished, and per-tile figures (issue to consumer start, consumer
start to release).
"""
import sys
import warnings

import numpy as np

KINDS = ["qkv", "attn", "o", "gu", "down"]
TILE_KINDS = {0: "qkv", 1: "o", 2: "gu", 3: "down", 4: "lm"}


def load(path):
    f = open(path, "rb").read()
    G, S = (int(v) for v in np.frombuffer(f[:8], dtype=np.int32))
    off = 8
    tl = np.frombuffer(f[off:off + G * S * 8], dtype=np.uint64).reshape(G, S).astype(np.float64)
    off += G * S * 8
    tiles = None
    if len(f) > off:
        mt = int(np.frombuffer(f[off:off + 4], dtype=np.int32)[0])
        off += 4
        tt = np.frombuffer(f[off:off + G * mt * 24], dtype=np.uint64).reshape(G, mt, 3).astype(np.float64)
        off += G * mt * 24
        tb = np.frombuffer(f[off:off + G * mt * 8], dtype=np.int32).reshape(G, mt, 2)
        tiles = (tt, tb)
    return G, S, tl, tiles


def summarise(path):
    G, S, tl, tiles = load(path)
    L = (S - 6) // 8 // 5
    g0, c0, g1, c1 = tl[:, S - 6], tl[:, S - 5], tl[:, S - 4], tl[:, S - 3]
    rate = (g1 - g0) / (c1 - c0)  # ns per SM clock, per CTA

    def to_ns(v, cta=slice(None)):
        return np.where(v > 0, g0[cta] + (v - c0[cta]) * rate[cta], np.nan)

    t0 = np.nanmin(to_ns(tl[:, 0]))
    out = [f"CTAs {G}, layers {L}, SM clock {1 / np.median(rate):.3f} GHz, "
           f"kernel {(np.nanmax(to_ns(tl[:, S - 1])) - t0) / 1e3:.1f} us"]
    agg = {}
    prev = 0.0
    for s in range(5 * L + 1):
        kind = "lm" if s == 5 * L else KINDS[s % 5]
        reg = to_ns(tl[:, 8 * s + 2]) - t0
        done = to_ns(tl[:, S - 2] if s == 5 * L else tl[:, 8 * s + 6]) - t0
        with np.errstate(all="ignore"):
            row = (np.nanmax(done) - prev,
                   np.nanmedian(reg) - prev if np.isfinite(reg).any() else np.nan,
                   np.nanmedian(done) - prev)
        agg.setdefault(kind, []).append(row)
        prev = np.nanmax(done)
    out.append("stage  count  span us  median in-registers us  median done us  total us")
    for kind in KINDS + ["lm"]:
        v = np.array(agg[kind])
        with np.errstate(all="ignore"):
            out.append(f"{kind:5s} {len(v):6d} {np.nanmean(v[:, 0]) / 1e3:8.2f} {np.nanmean(v[:, 1]) / 1e3:23.2f} "
                       f"{np.nanmean(v[:, 2]) / 1e3:15.2f} {np.nansum(v[:, 0]) / 1e3:9.1f}")
    if tiles is not None:
        tt, tb = tiles
        stat = {}
        for c in range(G):
            for j in range(tt.shape[1]):
                if tt[c, j, 0] == 0:
                    continue
                kind = TILE_KINDS.get((int(tb[c, j, 1]) >> 12) & 0xF, "?")
                iss, land, rel = (to_ns(tt[c, j, k], c) for k in range(3))
                stat.setdefault(kind, []).append((land - iss, rel - land, int(tb[c, j, 1]) & 0xFFF))
        out.append("tiles  count  rows/tile  issued->consumer start us  consumer start->released us")
        for kind in ["qkv", "o", "gu", "down", "lm"]:
            if kind in stat:
                v = np.array(stat[kind], dtype=np.float64)
                out.append(f"{kind:5s} {len(v):6d} {np.mean(v[:, 2]):10.1f} {np.nanmean(v[:, 0]) / 1e3:26.2f} "
                           f"{np.nanmean(v[:, 1]) / 1e3:28.2f}")
    return "\n".join(out)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python -m sqb200.timeline <timeline file>")
    with warnings.catch_warnings():
        warnings.simplefilter("ignore", RuntimeWarning)  # stages some CTAs never stamp (attention)
        print(summarise(sys.argv[1]))
