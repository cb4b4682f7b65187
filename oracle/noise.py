"""CPU restatement of the sampler's noise source (test infrastructure only).

This module is the checker for the in-kernel Philox noise of ``qedge_b200``.
Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` import it; the product path never does.

The reference sampler draws its categorical sample with
``torch.multinomial`` on torch's global generator
(``src/compute/sampler.py:38`` and ``:40``), which is equivalent to an
exponential race ``argmax_j w_j / E_j`` with ``E ~ Exp(1)``.  The reference
has no per-request seed.  The B200 path keys its noise on
``(seed, step, row)`` with a Philox4x32-10 counter generator (Salmon et al.,
"Parallel random numbers: as easy as 1, 2, 3", SC'11; constants and round
function from that paper).  Known-answer vectors from the Random123
distribution pin :func:`philox4x32_10` (see ``tests/test_oracle_noise.py``).

The Exp(1) noise tensor ``E[B, V]`` is defined as a "minimum-first" tree,
which gives i.i.d. Exp(1) marginals and lets the GPU kernel skip generating
noise for tokens that cannot win the race:

* root (one per row): ``E_root = -ln(u_root) / V``; a uniformly chosen token
  ``s`` carries that minimum;
* group ``G`` (up to 32 tokens, layout below, global group id ``g``): its
  minimum ``E_min(G) = E_root + (-ln(u_m)) / n_G`` where ``u_m`` is word
  ``g mod 4`` of one Philox call with counter ``g // 4`` (tag 3: one call
  serves four consecutive groups, so the kernel can bound every group cheaply),
  carried by member ``select(y, n_G)`` -- or ``E_root`` carried by ``s`` if
  ``s`` is in ``G``; then the second smallest value
  ``E2(G) = E_min(G) + (-ln(u_z)) / (n_G - 1)`` carried by member
  ``select(w, n_G - 1)`` counted among the members other than the argmin,
  where ``(y, z, w)`` are words of one Philox call whose counter is ``g``
  (tag 1; word ``x`` is unused);
* every other token ``j`` of ``G``: ``E_j = E2(G) + (-ln(u_j))``.

By the memoryless property of the exponential distribution this is exactly
the joint law of ``V`` i.i.d. Exp(1) variables.  All arithmetic below is
IEEE float32 with round-to-nearest and no fused multiply-add, so the CUDA
kernel (which uses ``__fadd_rn``/``__fmul_rn``/``__fdiv_rn``) produces the
same bits.
"""
from __future__ import annotations

import numpy as np

# Philox4x32 multipliers and Weyl key increments (Salmon et al. 2011).
PHILOX_M0 = 0xD2511F53
PHILOX_M1 = 0xCD9E8D57
PHILOX_W0 = 0x9E3779B9
PHILOX_W1 = 0xBB67AE85

TAG_ROOT, TAG_GROUP, TAG_TOKEN, TAG_GMIN = 0, 1, 2, 3
NSLICE = 16         # canonical vocab slices per row (also the max vocab-shard count)
TILE = 1024         # ids per tile inside a slice
GROUP_LANES = 32    # groups per tile

_MASK32 = np.uint64(0xFFFFFFFF)


def _f32(bits: int) -> np.float32:
    return np.array([bits], dtype=np.uint32).view(np.float32)[0]


# float32 constants, given by bit pattern so C and numpy agree exactly.
F_SQRT2 = _f32(0x3FB504F3)     # 1.41421353816986083984375
F_C3 = _f32(0x3F2AAAAB)        # 2/3
F_C5 = _f32(0x3ECCCCCD)        # 2/5
F_C7 = _f32(0x3E924925)        # 2/7
F_C9 = _f32(0x3E638E39)        # 2/9
F_LN2_HI = _f32(0x3F317200)    # 0.693145751953125 (15 significant bits)
F_LN2_LO = _f32(0x35BFBE8E)    # ln 2 - LN2_HI
F_2M24 = _f32(0x33800000)      # 2^-24


def philox4x32_10(c0, c1, c2, c3, k0, k1):
    """Vectorised Philox4x32 with 10 rounds.  All inputs are uint32 arrays
    (broadcastable) or ints; returns four uint32 arrays."""
    c = [np.asarray(x, dtype=np.uint64) for x in (c0, c1, c2, c3)]
    c = np.broadcast_arrays(*c)
    c = [x.copy() for x in c]
    k0 = np.uint64(int(k0) & 0xFFFFFFFF)
    k1 = np.uint64(int(k1) & 0xFFFFFFFF)
    m0, m1 = np.uint64(PHILOX_M0), np.uint64(PHILOX_M1)
    s32 = np.uint64(32)
    for _ in range(10):
        p0 = m0 * c[0]
        p1 = m1 * c[2]
        hi0, lo0 = p0 >> s32, p0 & _MASK32
        hi1, lo1 = p1 >> s32, p1 & _MASK32
        c = [hi1 ^ c[1] ^ k0, lo1, hi0 ^ c[3] ^ k1, lo0]
        k0 = (k0 + np.uint64(PHILOX_W0)) & _MASK32
        k1 = (k1 + np.uint64(PHILOX_W1)) & _MASK32
    return [x.astype(np.uint32) for x in c]


def uniform_open(w) -> np.ndarray:
    """Map a 32-bit word to an odd multiple of 2^-24 in (0, 1): exact in fp32."""
    w = np.asarray(w, dtype=np.uint32)
    odd = ((w >> np.uint32(9)) * np.uint32(2) + np.uint32(1)).astype(np.float32)
    return (odd * F_2M24).astype(np.float32)


def neglog_f32(u) -> np.ndarray:
    """-ln(u) for u in [2^-24, 1), float32, round-to-nearest, no FMA.

    Argument reduction u = m * 2^e with m in [sqrt(1/2), sqrt(2)], then
    ln m = 2 atanh(f), f = (m-1)/(m+1), summed as the odd series
    2(f + f^3/3 + f^5/5 + f^7/7 + f^9/9) (|f| <= 0.1716, truncation < 1e-8
    relative).  ln 2 is split into a 15-bit head and a tail so e*ln2 is exact.
    """
    u = np.asarray(u, dtype=np.float32)
    bits = u.view(np.uint32)
    e = (bits >> np.uint32(23)).astype(np.int32) - 127
    m = ((bits & np.uint32(0x7FFFFF)) | np.uint32(0x3F800000)).view(np.float32)
    big = m > F_SQRT2
    m = np.where(big, m * np.float32(0.5), m).astype(np.float32)
    e = np.where(big, e + 1, e)
    one = np.float32(1.0)
    f = ((m - one) / (m + one)).astype(np.float32)
    f2 = (f * f).astype(np.float32)
    t = (f2 * F_C9).astype(np.float32)
    t = (F_C7 + t).astype(np.float32)
    t = (f2 * t).astype(np.float32)
    t = (F_C5 + t).astype(np.float32)
    t = (f2 * t).astype(np.float32)
    t = (F_C3 + t).astype(np.float32)
    poly = (f2 * t).astype(np.float32)
    lnm = ((f + f) + (f * poly).astype(np.float32)).astype(np.float32)
    ef = e.astype(np.float32)
    r = (ef * F_LN2_HI).astype(np.float32) + ((ef * F_LN2_LO).astype(np.float32) + lnm).astype(np.float32)
    return (-r.astype(np.float32)).astype(np.float32)


def slice_starts(V: int) -> np.ndarray:
    """Canonical slice boundaries: NSLICE contiguous slices whose starts are
    multiples of 8 ids (16-byte aligned for bf16/fp16 rows); the last slice
    ends at V."""
    s = [((g * V) // (NSLICE * 8)) * 8 for g in range(NSLICE)] + [V]
    return np.array(s, dtype=np.int64)


def group_layout(V: int):
    """For every token id return (global group id, member index) and the
    member count of every group.

    Inside slice g (ids [start, end)), the local offset o = j - start splits
    as tile t = o >> 10, block b = (o >> 8) & 3, lane l = (o >> 3) & 31,
    element i = o & 7; the token belongs to local group t*32 + l and is member
    number b*8 + i of it (members are numbered in increasing id order).
    """
    starts = slice_starts(V)
    gid = np.empty(V, dtype=np.int64)
    mem = np.empty(V, dtype=np.int64)
    sizes = []
    base = 0
    for g in range(NSLICE):
        a, z = int(starts[g]), int(starts[g + 1])
        L = z - a
        ntiles = (L + TILE - 1) // TILE
        o = np.arange(L, dtype=np.int64)
        t = o >> 10
        b = (o >> 8) & 3
        lane = (o >> 3) & 31
        i = o & 7
        gid[a:z] = base + t * GROUP_LANES + lane
        mem[a:z] = b * 8 + i
        cnt = np.bincount(t * GROUP_LANES + lane, minlength=ntiles * GROUP_LANES)
        sizes.append(cnt)
        base += ntiles * GROUP_LANES
    sizes = np.concatenate(sizes) if sizes else np.zeros(0, np.int64)
    return gid, mem, sizes.astype(np.int64)


def _select(w1, w2, n):
    """floor(((w1 << 32) | w2) * n / 2^64) for n < 2^24 (exact, uint64 math)."""
    w1 = np.asarray(w1, dtype=np.uint64)
    w2 = np.asarray(w2, dtype=np.uint64)
    n = np.asarray(n, dtype=np.uint64)
    s32 = np.uint64(32)
    return ((w1 * n + ((w2 * n) >> s32)) >> s32).astype(np.int64)


def _select32(w, n):
    """floor(w * n / 2^32) for n <= 2^24."""
    return ((np.asarray(w, dtype=np.uint64) * np.asarray(n, dtype=np.uint64)) >> np.uint64(32)).astype(np.int64)


def philox_noise(B: int, V: int, seed: int, step: int, row_offset: int = 0) -> np.ndarray:
    """Materialise the Exp(1) noise tensor E[B, V] that the kernel's Philox
    mode uses for rows row_offset .. row_offset+B-1."""
    assert 0 < V < (1 << 24)
    k0, k1 = seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF
    s_lo = step & 0xFFFFFFFF
    hi = ((step >> 32) << 2) & 0xFFFFFFFF
    gid, mem, sizes = group_layout(V)
    NG = sizes.shape[0]
    Vf = np.float32(V)
    out = np.empty((B, V), dtype=np.float32)
    jarange = np.arange(V, dtype=np.int64)
    garange = np.arange(NG, dtype=np.int64)
    n = np.maximum(sizes, 1)
    nf = n.astype(np.float32)
    n1f = np.maximum(n - 1, 1).astype(np.float32)
    for r in range(B):
        row = row_offset + r
        w = philox4x32_10(0, row, s_lo, hi | TAG_ROOT, k0, k1)
        e_root = (neglog_f32(uniform_open(w[0])) / Vf).astype(np.float32)
        s = int(_select(w[1], w[2], V))
        wg = philox4x32_10(garange, row, s_lo, hi | TAG_GROUP, k0, k1)
        wq = philox4x32_10(garange >> 2, row, s_lo, hi | TAG_GMIN, k0, k1)
        umin = np.choose((garange & 3).astype(np.int64), wq)
        e_min = (e_root + (neglog_f32(uniform_open(umin)) / nf).astype(np.float32)).astype(np.float32)
        arg = _select32(wg[1], n)
        gs = gid[s]
        e_min[gs] = e_root
        arg[gs] = mem[s]
        e2 = (e_min + (neglog_f32(uniform_open(wg[2])) / n1f).astype(np.float32)).astype(np.float32)
        i2 = _select32(wg[3], np.maximum(n - 1, 1))
        arg2 = np.where(i2 < arg, i2, i2 + 1)
        single = n < 2
        e2[single] = np.inf
        arg2[single] = -1
        wt = philox4x32_10(jarange >> 2, row, s_lo, hi | TAG_TOKEN, k0, k1)
        wsel = np.choose((jarange & 3).astype(np.int64), wt)
        e2_j = e2[gid]
        with np.errstate(invalid="ignore"):
            e = (e2_j + neglog_f32(uniform_open(wsel))).astype(np.float32)
        is2 = mem == arg2[gid]
        e[is2] = e2_j[is2]
        is_arg = mem == arg[gid]
        e[is_arg] = e_min[gid][is_arg]
        out[r] = e
    return out
