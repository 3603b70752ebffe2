"""Seeded weights for the configuration-2-shaped whole-model golden trace.

The reference's own initialiser would have to run wherever the test runs, and
storing configuration 2's weights (a 50,257 x 128 embedding alone is 25 MB)
would bloat the fixtures.  Instead both the golden generator (which runs the
reference model) and the GPU test (which runs this package's model) load the
same weights, drawn here from a seeded numpy generator in state-dict order.
"""

from __future__ import annotations

import numpy as np

VOCAB, MAX_LEN, LAYOUT, WIDTH, HEADS, SLOTS, READS, WRITES, MEMORY_HEADS = 50257, 512, "BBBBBBBA", 128, 4, 256, 16, 4, 1


def model_kwargs() -> dict:
    return dict(vocab_size=VOCAB, maximum_sequence_length=MAX_LEN, layout=LAYOUT, width=WIDTH, heads=HEADS,
                slots=SLOTS, reads=READS, writes=WRITES, memory_heads=MEMORY_HEADS)


def seeded_params(shapes: dict[str, tuple[int, ...]], seed: int = 2) -> dict[str, np.ndarray]:
    """One float32 array per parameter name: vectors near 1 (scales) or near 0
    (biases), matrices and tensors with entries of size 1/sqrt(fan-in)."""
    rng = np.random.default_rng(seed)
    out = {}
    for name in sorted(shapes):
        shape = tuple(shapes[name])
        if len(shape) <= 1:
            base = 1.0 if name.endswith("weight") or name.endswith("scale") else 0.0
            out[name] = (base + 0.05 * rng.standard_normal(shape)).astype(np.float32)
        else:
            fan_in = int(np.prod(shape[1:]))
            out[name] = (rng.standard_normal(shape) / np.sqrt(fan_in)).astype(np.float32)
    return out
