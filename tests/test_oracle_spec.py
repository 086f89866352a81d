"""Self-consistency checks of the oracle's restatement of the ASTC rules."""
import numpy as np
import pytest

from oracle import oracle as O

LEVELS = [2, 3, 4, 5, 6, 8, 10, 12, 16, 20, 24, 32, 40, 48, 64, 80, 96, 128, 160, 192, 256]


@pytest.mark.parametrize("q", range(4, 21))
def test_color_unquantisation_is_a_permutation_of_even_levels(q):
    vals = sorted(O.lib().astc_oracle_unquant_color(q, v) for v in range(LEVELS[q]))
    ideal = [round(i * 255 / (LEVELS[q] - 1)) for i in range(LEVELS[q])]
    assert max(abs(a - b) for a, b in zip(vals, ideal)) <= 1
    assert vals[0] == 0 and vals[-1] == 255 and len(set(vals)) == LEVELS[q]


@pytest.mark.parametrize("q", range(0, 12))
def test_weight_unquantisation_is_a_permutation_of_even_levels(q):
    vals = sorted(O.lib().astc_oracle_unquant_weight(q, v) for v in range(LEVELS[q]))
    ideal = [round(i * 64 / (LEVELS[q] - 1)) for i in range(LEVELS[q])]
    assert max(abs(a - b) for a, b in zip(vals, ideal)) <= 1
    assert vals[0] == 0 and vals[-1] == 64


def test_bise_bit_counts():
    f = O.lib().astc_oracle_bise_bits
    assert f(5, 1) == 8          # five trits, no extra bits
    assert f(3, 3) == 7          # three quints
    assert f(36, 2) == 72        # 2-bit plain values
    assert f(18, 20) == 144
    assert f(7, 4) == 7 + 12     # trit + 1 bit: 7 + ceil(56/5)


def test_fp16_rule_round_toward_zero():
    f = O.lib().astc_oracle_unorm16_to_half
    assert f(0xFFFF) == 0x3C00
    assert f(0) == 0
    for c in [1, 2, 3, 4, 5, 100, 2047, 2048, 2049, 30000, 65534]:
        h = np.array([f(c)], np.uint16).view(np.float16)[0]
        exact = c / 65536.0
        assert float(h) <= exact < float(np.nextafter(h, np.float16(np.inf)))


def test_partition_function_spreads_and_is_deterministic():
    f = O.lib().astc_oracle_partition
    for count in (2, 3, 4):
        seen = set()
        for seed in range(1024):
            parts = {f(seed, x, y, count, 0) for x in range(6) for y in range(6)}
            assert max(parts) < count
            seen |= parts
        assert seen == set(range(count))


def test_error_colour_for_reserved_and_void_extent_rules():
    blk = np.zeros(16, np.uint8)  # block mode 0 is reserved
    t = O.decode_blocks(blk, 6, O.OUT_UNORM8)
    assert np.all(t[..., 0] == 255) and np.all(t[..., 1] == 0) and np.all(t[..., 2] == 255) and np.all(t[..., 3] == 255)
    # Constant LDR void-extent: mode 0x1FC, reserved bits set, all-ones extents.
    v = np.zeros(16, np.uint8)
    bits = 0xDFC | (0x1FFF << 12) | (0x1FFF << 25) | (0x1FFF << 38) | (0x1FFF << 51)
    v[:8] = np.frombuffer(int(bits).to_bytes(8, "little"), np.uint8)
    v[8:] = np.frombuffer(np.array([0x1234, 0x8000, 0xFFFF, 0x0001], "<u2").tobytes(), np.uint8)
    t16 = O.decode_blocks(v, 4, O.OUT_UNORM16)
    assert np.all(t16[..., 0] == 0x1234) and np.all(t16[..., 2] == 0xFFFF)
    # HDR void-extent in the LDR profile -> error colour.
    h = v.copy()
    h[1] |= 0x02  # bit 9
    assert np.all(O.decode_blocks(h, 4, O.OUT_UNORM8)[..., 1] == 0)
