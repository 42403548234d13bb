"""Conversions between the two DeltaNet conv-state layouts of the reference.

The context keeps the C++ core's layout: a ring of the kernel_size - 1 past inputs per channel,
[C][K-1], with `conv_pos` the slot of the oldest (core/cpu_ops.cpp:89-129; qwen3_5.h:158-162).
The hybrid v2 export keeps a shift register [C][K] that already holds the current input: each
step forms cat(state[:, 1:], x) and convolves all K entries (export_hybrid_chunks.py:115-117), so
its first column is dropped before it is ever used again.  Both give the same convolution of the
same K inputs; these helpers move a sequence's state between the two (host numpy arrays, e.g.
around `Context.deltanet_state_export / _import`)."""
import numpy as np


def conv_ring_to_shift(conv: np.ndarray, conv_pos: int) -> np.ndarray:
    """[C][K-1] ring with the oldest input at `conv_pos` -> [C][K] shift register whose columns
    1..K-1 are the K-1 past inputs oldest first; column 0 (never read again) is zero."""
    C, L = conv.shape
    order = [(conv_pos + j) % L for j in range(L)]
    shift = np.zeros((C, L + 1), dtype=conv.dtype)
    shift[:, 1:] = conv[:, order]
    return shift


def conv_shift_to_ring(shift: np.ndarray):
    """[C][K] shift register -> ([C][K-1] ring, conv_pos = 0): the last K-1 columns, oldest first."""
    return np.ascontiguousarray(shift[:, 1:]), 0
