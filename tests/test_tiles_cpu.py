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


# native G64 records: one {scale, bias} pair per row and 64 inputs
G64_SHAPES = [  # experts, out, in, tile_rows, gate/up pair
    (3, 40, 128, 16, True),
    (2, 70, 192, 32, False),     # ragged: the last chunk holds one group of 64
    (2, 24, 64, 16, False),
    (1, 512, 2048, 16, True),
    (1, 2048, 512, 32, False),
]


@pytest.mark.parametrize("E,out,inn,tr,pair", G64_SHAPES)
def test_g64_round_trip(E, out, inn, tr, pair):
    rng = np.random.default_rng(E * out + inn + 64)
    a = O.make_q4_bank(rng, E, out, inn, 64)
    b = O.make_q4_bank(rng, E, out, inn, 64) if pair else None
    rec = O.tile_records(a, b, tr, 64)
    back = O.untile_records(rec, E, out, inn, 2 if pair else 1, tr, 64)
    for bank, (w, s, bb) in zip([a] + ([b] if pair else []), back):
        np.testing.assert_array_equal(w, bank.w)
        np.testing.assert_array_equal(s, O.bf16_bits(bank.scales))
        np.testing.assert_array_equal(bb, O.bf16_bits(bank.biases))


@pytest.mark.parametrize("E,out,inn,tr,pair", G64_SHAPES[:3])
def test_g64_lane_addressing(E, out, inn, tr, pair):
    """The words sit where they do in groups of 32 (1024 bytes per (p, m));
    the 128 bytes of scales per (p, m) hold, at (g*2 + cb)*8 + h*4, the
    {scale, bias} of row 16m+g+8h and group 2ch+cb - the one word the GEMV
    lane (g, c) reads for cb = c&1 and the GEMM reads per 64-input atom cb."""
    rng = np.random.default_rng(9)
    a = O.make_q4_bank(rng, E, out, inn, 64)
    b = O.make_q4_bank(rng, E, out, inn, 64) if pair else None
    banks = [a] + ([b] if pair else [])
    NP, MT = len(banks), tr // 16
    RB, nch, G, W = -(-out // tr), -(-inn // 128), inn // 64, inn // 8
    rec = O.tile_records(a, b, tr, 64).reshape(E, RB, nch, NP * MT * 1152)
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
                                cb = c & 1
                                soff = NP * MT * 1024 + (p * MT + m) * 128 + (g * 2 + cb) * 8 + h * 4
                                sv = r[soff:soff + 4].view(np.uint16)
                                gi = 2 * ch + cb
                                ok = row < out and gi < G
                                assert sv[0] == (sbits[p][e, row, gi] if ok else 0)
                                assert sv[1] == (bbits[p][e, row, gi] if ok else 0)


def test_g64_records_carry_the_expanded_banks():
    """Untiling native G64 records and repeating each pair for both halves
    gives exactly the group-32 records' content of the expanded bank."""
    rng = np.random.default_rng(5)
    a = O.make_q4_bank(rng, 2, 48, 320, 64)
    x = O.Q4Bank(a.w, np.repeat(a.scales, 2, axis=-1), np.repeat(a.biases, 2, axis=-1))
    w64, s64, b64 = O.untile_records(O.tile_records(a, None, 16, 64), 2, 48, 320, 1, 16, 64)[0]
    w32, s32, b32 = O.untile_records(O.tile_records(x, None, 16), 2, 48, 320, 1, 16)[0]
    np.testing.assert_array_equal(w64, w32)
    np.testing.assert_array_equal(np.repeat(s64, 2, axis=-1), s32)
    np.testing.assert_array_equal(np.repeat(b64, 2, axis=-1), b32)


def test_library_reports_the_g64_pool_size():
    import vxmoe._lib as L
    lib = L.load()
    for E, out, inn, tr, pair in G64_SHAPES:
        rng = np.random.default_rng(2)
        a = O.make_q4_bank(rng, E, out, inn, 64)
        b = O.make_q4_bank(rng, E, out, inn, 64) if pair else None
        assert lib.vx_q4_tiles_bytes_group(E, out, inn, 2 if pair else 1, tr, 64) == \
            O.tile_records(a, b, tr, 64).nbytes
    # groups of 32 through the same call
    assert lib.vx_q4_tiles_bytes_group(3, 40, 96, 2, 16, 32) == lib.vx_q4_tiles_bytes(3, 40, 96, 2, 16)
    # the C2 layer natively: 1024 + 128 bytes per 16 rows x 128 inputs
    assert lib.vx_q4_tiles_bytes_group(512, 512, 2048, 2, 16, 64) == \
        2 * 512 * 512 * (2048 // 8 * 4 + 2048 // 64 * 4)
    assert lib.vx_q4_tiles_bytes_group(4, 64, 96, 1, 16, 64) == 0    # in not a multiple of 64
    assert lib.vx_q4_tiles_bytes_group(4, 64, 128, 1, 16, 48) == 0   # only groups of 32 and 64
    assert lib.vx_q4_tiles_bytes_group(4, 64, 128, 1, 16, 128) == 0
