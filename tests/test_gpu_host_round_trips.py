"""Zero per-token host round trips, shown by the device's own activity record.

The engine's CUDA runtime is linked statically, so a host-API interposer
would not see its calls; CUPTI's activity records (through torch.profiler)
cover every kernel, copy and memset the process's context executes, whoever
issued it.  Two engines with the same weights and the same prefilled cohort
each run one decode epoch, one with K = 1 and one with K = 8, under the
profiler: the device activity of the two epochs must be the same list --
one launch of the epoch kernel and the same few copies of the 8 inputs and
2 outputs -- although the second runs eight decoder steps (model calls 8 in
the control output, against 1).  Nothing in an epoch scales with K on the
host side of the boundary.
"""

from __future__ import annotations

from collections import Counter

import pytest

from scenario import decode_inputs, make_scenario, prefill_epochs

pytestmark = pytest.mark.gpu


def _device_activity(engine, inputs):
    import torch
    from torch.autograd import DeviceType
    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA]) as prof:
        out = engine.run(**inputs)
        torch.cuda.synchronize()
    names = Counter(e.name for e in prof.events() if e.device_type == DeviceType.CUDA)
    return out, names


def test_epoch_device_activity_does_not_grow_with_k(cuda_ok):
    from cruise_b200.engine import EpochEngine
    from cruise_b200.model_config import TINY

    activity = {}
    for k in (1, 8):
        engine = EpochEngine("tiny")
        engine.init_synthetic(0)
        # seed 5: every row decodes all 8 steps of the K = 8 epoch (no EOS on the way)
        sc = make_scenario(vocab=TINY.vocab, seed=5, active_rows=(1, 1, 1, 1), k=k, budget=(8, 8))
        for inputs in prefill_epochs(sc, TINY.block_size, TINY.vocab):
            assert engine.run(**inputs).status == 0
        out, names = _device_activity(engine, decode_inputs(sc, TINY.block_size))
        engine.close()
        assert out.status == 0 and int(out.control_out[4]) == k, (k, list(out.control_out[:6]))
        activity[k] = names
    epoch_kernels = {n: c for n, c in activity[8].items() if "resident_epoch_kernel" in n}
    assert list(epoch_kernels.values()) == [1], activity[8]
    assert activity[1] == activity[8], (activity[1], activity[8])
    assert sum(activity[8].values()) <= 8, activity[8]
