"""Pins of the noise oracle: Philox known answers, -ln accuracy, Exp(1) law."""
import numpy as np
from scipy import stats

from oracle import noise as N

# Known-answer vectors for Philox4x32-10 from the Random123 distribution
# (counter, key) -> output.
KAT = [
    ((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
    ((0xFFFFFFFF,) * 4, (0xFFFFFFFF,) * 2, (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
    ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
     (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
]


def test_philox_known_answers():
    for ctr, key, want in KAT:
        got = N.philox4x32_10(*ctr, *key)
        assert tuple(int(x) for x in got) == want


def test_neglog_accuracy():
    w = np.random.default_rng(0).integers(0, 2**32, 2_000_000, dtype=np.uint64).astype(np.uint32)
    u = N.uniform_open(w)
    assert u.min() > 0 and u.max() < 1
    got = N.neglog_f32(u).astype(np.float64)
    want = -np.log(u.astype(np.float64))
    assert np.max(np.abs(got - want) / np.maximum(want, 1e-30)) < 3e-7
    # extreme arguments
    for x in (2.0**-24, 1 - 2.0**-24, 0.5, 0.70710677):
        v = N.neglog_f32(np.array([x], np.float32))[0]
        assert abs(v + np.log(np.float32(x))) <= 3e-7 * max(1.0, abs(np.log(x)))


def test_group_layout_partitions_vocab():
    for V in (1, 7, 8, 1000, 1024, 4099, 248_320):
        gid, mem, sizes = N.group_layout(V)
        assert sizes.sum() == V
        assert np.all(np.bincount(gid, minlength=sizes.size) == sizes)
        # members are numbered 0..n-1 in increasing id order inside each group
        order = np.lexsort((np.arange(V), gid))
        ranks = np.arange(V) - np.searchsorted(gid[order], gid[order])
        assert np.all(mem[order] == ranks)


def test_group_order_statistics():
    """Inside every group the noise is minimum-first: one member holds the
    group minimum, one the second smallest value, and the gap between them
    is Exp(1)/(n-1); the second member is uniform among the others."""
    V = 248_320
    E = N.philox_noise(2, V, seed=77, step=3)
    gid, mem, sizes = N.group_layout(V)
    full = sizes[gid] == 32
    gaps, pos2 = [], []
    for r in range(2):
        e = E[r][full]
        g = gid[full]
        order = np.lexsort((e, g))
        eg, gg, mg = e[order], g[order], mem[full][order]
        first = np.r_[True, gg[1:] != gg[:-1]]
        idx = np.flatnonzero(first)
        gaps.append((eg[idx + 1] - eg[idx]) * 31.0)
        pos2.append(mg[idx + 1])
    gaps = np.concatenate(gaps)
    assert stats.kstest(gaps, "expon").pvalue > 1e-3
    counts = np.bincount(np.concatenate(pos2), minlength=32)
    assert stats.chisquare(counts).pvalue > 1e-3


def test_philox_noise_is_exp1():
    E = N.philox_noise(3, 248_320, seed=2024, step=9)
    for r in range(3):
        assert stats.kstest(E[r], "expon").pvalue > 1e-3
    assert abs(float(E.mean()) - 1.0) < 0.01
    # deterministic and keyed on (seed, step, row)
    E2 = N.philox_noise(1, 248_320, seed=2024, step=9, row_offset=1)
    np.testing.assert_array_equal(E[1], E2[0])
    E3 = N.philox_noise(1, 248_320, seed=2024, step=10)
    assert not np.array_equal(E[0], E3[0])


def test_philox_noise_minimum_tree():
    # the row minimum is carried by exactly one token and equals E_root
    E = N.philox_noise(4, 5000, seed=1, step=0)
    for r in range(4):
        assert np.sum(E[r] == E[r].min()) == 1
