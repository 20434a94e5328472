"""The tiled expert pool layout on the CPU: the oracle's record layout round
trips to the MLX arrays, places every word and scale where the decode
kernel's lanes read them, and has the size the library reports."""
from __future__ import annotations

import numpy as np
import pytest

import vxmoe_oracle as O

SHAPES = [  # experts, out, in, tile_rows, gate/up pair
    (3, 40, 96, 16, True),
    (2, 70, 160, 32, False),
    (2, 24, 32, 16, False),
    (1, 512, 2048, 16, True),
    (1, 2048, 512, 32, False),
]


@pytest.mark.parametrize("E,out,inn,tr,pair", SHAPES)
def test_round_trip(E, out, inn, tr, pair):
    rng = np.random.default_rng(E * out + inn)
    a = O.make_q4_bank(rng, E, out, inn)
    b = O.make_q4_bank(rng, E, out, inn) if pair else None
    rec = O.tile_records(a, b, tr)
    back = O.untile_records(rec, E, out, inn, 2 if pair else 1, tr)
    for bank, (w, s, bb) in zip([a] + ([b] if pair else []), back):
        np.testing.assert_array_equal(w, bank.w)
        np.testing.assert_array_equal(s, O.bf16_bits(bank.scales))
        np.testing.assert_array_equal(bb, O.bf16_bits(bank.biases))


@pytest.mark.parametrize("E,out,inn,tr,pair", SHAPES[:3])
def test_lane_addressing(E, out, inn, tr, pair):
    """Each lane (g, c) of the consuming warp finds, at the offsets the kernel
    uses, words 4c..4c+3 of rows 16m+g and 16m+g+8 and the scale/bias pairs of
    groups 4ch+2(c&1), +1; padding is zero."""
    rng = np.random.default_rng(7)
    a = O.make_q4_bank(rng, E, out, inn)
    b = O.make_q4_bank(rng, E, out, inn) if pair else None
    banks = [a] + ([b] if pair else [])
    NP, MT = len(banks), tr // 16
    RB, nch, G, W = -(-out // tr), -(-inn // 128), inn // 32, inn // 8
    rec = O.tile_records(a, b, tr).reshape(E, RB, nch, NP * MT * 1280)
    sbits = [O.bf16_bits(bk.scales) for bk in banks]
    bbits = [O.bf16_bits(bk.biases) for bk in banks]
    for e in range(E):
        for rb in range(RB):
            for ch in range(nch):
                r = rec[e, rb, ch]
                for p in range(NP):
                    for m in range(MT):
                        for lane in range(32):
                            g, c = lane >> 2, lane & 3
                            for h in range(2):
                                row = rb * tr + 16 * m + g + 8 * h
                                off = (p * MT + m) * 1024 + h * 512 + lane * 16
                                got = r[off:off + 16].view(np.uint32)
                                for j in range(4):
                                    wd = ch * 16 + 4 * c + j
                                    exp = banks[p].w[e, row, wd] if row < out and wd < W else 0
                                    assert got[j] == exp
                                soff = NP * MT * 1024 + (p * MT + m) * 256 + (g * 2 + (c & 1)) * 16
                                sv = r[soff + 8 * h:soff + 8 * h + 8].view(np.uint16)
                                ga = 4 * ch + 2 * (c & 1)
                                for j, (src, gg) in enumerate(((sbits, ga), (sbits, ga + 1),
                                                               (bbits, ga), (bbits, ga + 1))):
                                    exp = src[p][e, row, gg] if row < out and gg < G else 0
                                    assert sv[j] == exp


def test_library_reports_the_pool_size():
    import vxmoe._lib as L
    lib = L.load()
    for E, out, inn, tr, pair in SHAPES:
        rng = np.random.default_rng(1)
        a = O.make_q4_bank(rng, E, out, inn)
        b = O.make_q4_bank(rng, E, out, inn) if pair else None
        assert lib.vx_q4_tiles_bytes(E, out, inn, 2 if pair else 1, tr) == O.tile_records(a, b, tr).nbytes
    # the C2 layer: same bytes as the MLX arrays (no padding at these shapes)
    assert lib.vx_q4_tiles_bytes(512, 512, 2048, 2, 16) == 2 * 512 * 512 * (2048 // 8 * 4 + 2048 // 32 * 4)
    assert lib.vx_q4_tiles_bytes(512, 2048, 512, 1, 32) == 512 * 2048 * (512 // 8 * 4 + 512 // 32 * 4)
    # rejected layouts
    assert lib.vx_q4_tiles_bytes(4, 64, 64, 2, 32) == 0     # gate/up pairs use 16-row tiles
    assert lib.vx_q4_tiles_bytes(4, 64, 48, 1, 16) == 0     # in not a multiple of 32
    assert lib.vx_q4_tiles_bytes(0, 64, 64, 1, 16) == 0
