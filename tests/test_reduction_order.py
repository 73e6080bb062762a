"""The batched GEMV's exactness argument, checked on the CPU in float32.

The canonical row sum is a 32-lane xor butterfly (levels 16, 8, 4, 2, 1) over
the lanes' group terms. gemv_batched_kernel (molten_b200/csrc/gemv_batched.cu)
gives a lane a whole row instead and replays that butterfly by visiting the
groups in 5-bit bit-reversed order through five nested loops; with a K split
each of 2^k warps folds one subtree and the subtree sums are added in the same
tree order. Float addition commutes, so these must equal the butterfly bit for
bit -- this test restates both orders in numpy float32 and compares them.
"""
import numpy as np
import pytest

F = np.float32


def butterfly(terms):
    """Lane 0's value after v += shfl_xor(v, m) for m = 16, 8, 4, 2, 1."""
    v = [F(t) for t in terms]
    for m in (16, 8, 4, 2, 1):
        v = [F(v[l] + v[l ^ m]) for l in range(32)]
    return v[0]


def nested(terms, ks_log2=0):
    """The kernel's loop nest: visit s = i0 + 2 i1 + 4 i2 + 8 i3 + 16 i4 reads
    group g = 16 i0 + 8 i1 + 4 i2 + 2 i3 + i4; level d assigns on its first
    iteration and adds after. With a K split, part p fixes the top ks_log2
    visit digits; the parts' sums are then added pairwise (p, p ^ 1), ..."""
    ks = 1 << ks_log2
    parts = []
    for p in range(ks):
        s_lo = p << (5 - ks_log2)
        lo = [0] * 5
        hi = [2] * 5
        for d in range(1, 5):
            if d >= 5 - ks_log2:
                lo[d] = (s_lo >> d) & 1
                hi[d] = lo[d] + 1
        l5 = None
        for i4 in range(lo[4], hi[4]):
            l4 = None
            for i3 in range(lo[3], hi[3]):
                l3 = None
                for i2 in range(lo[2], hi[2]):
                    l2 = None
                    for i1 in range(lo[1], hi[1]):
                        l1 = None
                        for i0 in range(2):
                            g = 16 * i0 + 8 * i1 + 4 * i2 + 2 * i3 + i4
                            t = F(terms[g])
                            l1 = t if i0 == 0 else F(l1 + t)
                        l2 = l1 if i1 == lo[1] else F(l2 + l1)
                    l3 = l2 if i2 == lo[2] else F(l3 + l2)
                l4 = l3 if i3 == lo[3] else F(l4 + l3)
            l5 = l4 if i4 == lo[4] else F(l5 + l4)
        parts.append(l5)
    while len(parts) > 1:
        parts = [F(parts[2 * q] + parts[2 * q + 1]) for q in range(len(parts) // 2)]
    return parts[0]


def _cases():
    g = np.random.default_rng(7)
    out = []
    for _ in range(60):
        scale = 10.0 ** g.integers(-30, 30, size=32)
        out.append((g.standard_normal(32) * scale).astype(np.float32))
    # cancellation-heavy rows, signed zeros, idle groups (K < 2048 leaves +0)
    big = np.float32(3e38)
    out.append(np.array([big, -big] * 16, np.float32))
    out.append(np.array([0.0, -0.0] * 16, np.float32))
    out.append(np.array([-0.0] * 32, np.float32))
    t = g.standard_normal(32).astype(np.float32)
    t[24:] = 0.0
    out.append(t)
    out.append(np.array([1.0, 1e-8] * 16, np.float32))
    return out


@pytest.mark.parametrize("ks_log2", [0, 1, 2, 3])
def test_nested_bitreversed_order_equals_butterfly(ks_log2):
    for terms in _cases():
        # some cases overflow on purpose (inf, inf - inf): both orders must
        # still produce the same bits
        with np.errstate(over="ignore", invalid="ignore"):
            a = butterfly(terms)
            b = nested(terms, ks_log2)
        assert np.float32(a).view(np.uint32) == np.float32(b).view(np.uint32), (ks_log2, terms)


def test_plain_sequential_order_differs():
    """The check has teeth: a left-to-right sum is a different order and
    differs from the butterfly on some inputs."""
    g = np.random.default_rng(3)
    differs = 0
    for _ in range(200):
        terms = g.standard_normal(32).astype(np.float32)
        seq = F(0.0)
        for t in terms:
            seq = F(seq + t)
        differs += np.float32(seq).view(np.uint32) != np.float32(butterfly(terms)).view(np.uint32)
    assert differs > 0
