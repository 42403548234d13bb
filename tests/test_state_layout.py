"""The two DeltaNet conv-state layouts (ring + conv_pos of core/cpu_ops.cpp:89-129, shift
register of export_hybrid_chunks.py:115-117) hold the same information: starting from converted
states, the C++ core's conv1d_update (the oracle's restatement) and a numpy restatement of the
hybrid export's shift step give the same conv outputs, step after step, and the conversions
round-trip.  CPU only."""
import numpy as np

from anelm_b200.state_layout import conv_ring_to_shift, conv_shift_to_ring


def ring_step(conv, pos, x, w):
    """conv1d_update, kernel 4 (core/cpu_ops.cpp:94-110): oldest at pos, then pos+1, pos+2."""
    p0, p1, p2 = pos, (pos + 1) % 3, (pos + 2) % 3
    y = conv[:, p0] * w[:, 0] + conv[:, p1] * w[:, 1] + conv[:, p2] * w[:, 2] + x * w[:, 3]
    conv[:, p0] = x
    return y, (pos + 1) % 3


def shift_step(state, x, w):
    """export_hybrid_chunks.py:115-116: new = cat(state[:, 1:], x); out = sum(new * w)."""
    new = np.concatenate([state[:, 1:], x[:, None]], axis=1)
    return (new * w).sum(axis=1), new


def test_ring_and_shift_layouts_give_the_same_convolution():
    rng = np.random.default_rng(3)
    C = 96
    w = rng.standard_normal((C, 4)).astype(np.float32)
    ring = rng.standard_normal((C, 3)).astype(np.float32)
    pos = 2
    shift = conv_ring_to_shift(ring, pos)
    for _ in range(7):
        x = rng.standard_normal(C).astype(np.float32)
        y_ring, pos = ring_step(ring, pos, x, w)
        y_shift, shift = shift_step(shift, x, w)
        np.testing.assert_allclose(y_ring, y_shift, rtol=1e-6, atol=1e-6)
    # converting back at any point continues the same sequence of outputs
    ring2, pos2 = conv_shift_to_ring(shift)
    x = rng.standard_normal(C).astype(np.float32)
    y_a, _ = ring_step(ring, pos, x, w)
    y_b, _ = ring_step(ring2.copy(), pos2, x, w)
    np.testing.assert_allclose(y_a, y_b, rtol=1e-6, atol=1e-6)


def test_round_trip_is_exact():
    rng = np.random.default_rng(4)
    ring = rng.standard_normal((10, 3)).astype(np.float32)
    for pos in range(3):
        back, p = conv_shift_to_ring(conv_ring_to_shift(ring, pos))
        order = [(pos + j) % 3 for j in range(3)]
        np.testing.assert_array_equal(back, ring[:, order])
        assert p == 0
