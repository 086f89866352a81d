"""The product's host-built decode tables against the oracle's rules."""
import ctypes as ct

import numpy as np

from oracle import oracle as O

LEVELS = [2, 3, 4, 5, 6, 8, 10, 12, 16, 20, 24, 32, 40, 48, 64, 80, 96, 128, 160, 192, 256]


def tables():
    from astc_kv_cuda.ops import host_tables
    raw = np.frombuffer(host_tables(), np.uint8)
    off = 0

    def take(dtype, shape):
        nonlocal off
        n = int(np.prod(shape)) * np.dtype(dtype).itemsize
        a = raw[off:off + n].view(dtype).reshape(shape)
        off += n
        return a
    t = {}
    t["mode"] = take(np.uint32, (3, 2048))
    t["part"] = take(np.uint32, (3, 3, 1024, 4))
    t["trit"] = take(np.uint16, (256,))
    t["quint"] = take(np.uint16, (128,))
    t["cunq"] = take(np.uint8, (21, 256))
    t["wunq"] = take(np.uint8, (12, 32))
    t["cquant"] = take(np.uint8, (10, 128))
    t["shape"] = take(np.uint8, (21,))
    off += off & 1
    t["dig3"] = take(np.uint16, (384,))
    t["infill"] = take(np.uint16, (3, 7, 7, 64))
    off = (off + 15) // 16 * 16
    t["sep"] = take(np.uint16, (3, 7, 8))
    assert (off + 15) // 16 * 16 == raw.size
    return t


def test_unquant_tables_match_oracle():
    t = tables()
    L = O.lib()
    for q in range(4, 21):
        for v in range(LEVELS[q]):
            assert t["cunq"][q][v] == L.astc_oracle_unquant_color(q, v)
    for q in range(12):
        for v in range(LEVELS[q]):
            assert t["wunq"][q][v] == L.astc_oracle_unquant_weight(q, v)


def test_partition_tables_match_oracle():
    t = tables()
    L = O.lib()
    for f, bs in enumerate((4, 6, 8)):
        small = int(bs * bs < 31)
        for count in (2, 3, 4):
            for seed in range(0, 1024, 7):
                words = t["part"][f][count - 2][seed]
                for y in range(bs):
                    for x in range(bs):
                        i = y * bs + x
                        got = (int(words[i >> 4]) >> (2 * (i & 15))) & 3
                        assert got == L.astc_oracle_partition(seed, x, y, count, small), (bs, count, seed, x, y)


def test_mode_table_validity_matches_oracle():
    """A mode is valid in the table iff the oracle decodes a block with that
    mode (1 partition, CEM 0) without reporting the error colour for
    reasons of the mode itself."""
    t = tables()
    for f, bs in enumerate((4, 6, 8)):
        for m in range(2048):
            if (m & 0x1FF) == 0x1FC:
                assert t["mode"][f][m] == 0
                continue
            blk = np.zeros(16, np.uint8)
            blk[0] = m & 0xFF
            blk[1] = (m >> 8) & 0x7
            info = O.block_info(blk, bs)
            entry = int(t["mode"][f][m])
            if entry & 1:
                # valid mode: the oracle may still reject for colour bits, but
                # the weight grid must agree when it decodes
                if info["kind"] == 0:
                    assert (info["wx"], info["wy"]) == ((entry >> 6) & 15, (entry >> 10) & 15)
                    assert info["dual"] == (entry >> 1) & 1
                    assert info["wq"] == (entry >> 2) & 15
            else:
                assert info["kind"] == 1, (bs, m)


def test_trit_quint_tables_cover_all_digit_tuples():
    t = tables()
    trits = {tuple((int(v) >> (2 * j)) & 3 for j in range(5)) for v in t["trit"]}
    quints = {tuple((int(v) >> (3 * j)) & 7 for j in range(3)) for v in t["quint"]}
    assert len(trits) == 243 and all(max(x) <= 2 for x in trits)
    assert len(quints) == 125 and all(max(x) <= 4 for x in quints)


def test_separable_infill_matches_texel_taps():
    """The per-axis taps (row evaluator) compose to the per-texel taps, both
    follow the spec's grid coordinates, and a full grid maps to itself."""
    t = tables()
    for f, bs in enumerate((4, 6, 8)):
        ds = (1024 + bs // 2) // (bs - 1)
        for n in range(2, bs + 1):
            for c in range(bs):
                g = (ds * c * (n - 1) + 32) >> 6
                e = int(t["sep"][f, n - 2, c])
                j, j1, frac = e & 15, (e >> 4) & 15, e >> 8
                assert (j, frac) == (g >> 4, g & 15)
                assert j1 == min(j + 1, 7) and j <= n - 1
                assert frac == 0 or j + 1 <= n - 1  # the upper tap is inside the grid when it has weight
                if n == bs:
                    assert (j, frac) == (c, 0)
        for wx in range(2, bs + 1):
            for wy in range(2, bs + 1):
                for y in range(bs):
                    for x in range(bs):
                        ex, ey = int(t["sep"][f, wx - 2, x]), int(t["sep"][f, wy - 2, y])
                        tap = int(t["infill"][f, wx - 2, wy - 2, y * bs + x])
                        assert tap == ((ex & 15) + (ey & 15) * wx) | ((ex >> 8) << 6) | ((ey >> 8) << 10)
