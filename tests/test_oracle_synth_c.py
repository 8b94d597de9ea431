"""The C restatement of the seeded weight generator (oracle/csynth.c) gives
the bits of the numpy one (oracle/synth.py), which the device generator is
pinned to by the GPU tests; full-depth oracle models are built with it."""

from __future__ import annotations

import numpy as np
import torch

from oracle.model import TINY, seeded_weights
from oracle.synth import synth_bf16_bits, synth_bf16_bits_c


def test_c_generator_equals_numpy_generator_on_offsets_and_seeds():
    for seed, tid, start, count in ((0, 0, 0, 4097), (3, 17, 123_456_789, 10_001), (2**40 + 5, 337, 7, 65_536)):
        expect = synth_bf16_bits(seed, tid, count, start=start)
        for threads in (1, 3):
            got = synth_bf16_bits_c(seed, tid, count, start=start, threads=threads)
            assert np.array_equal(got, expect), (seed, tid, start, threads)


def test_c_generator_builds_the_same_tiny_model():
    slow = seeded_weights(TINY, seed=0)
    fast = seeded_weights(TINY, seed=0, use_c=True)
    assert slow.keys() == fast.keys()
    for name in slow:
        assert torch.equal(slow[name].view(torch.int16), fast[name].view(torch.int16)), name
