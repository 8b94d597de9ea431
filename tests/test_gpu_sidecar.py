"""The out-of-process sidecar on the GPU: the same plans through the sidecar
(server process) and through the in-process bridge give the same tokens,
generations, statuses and import proofs -- plain epochs, a host-snapshot import
and a device-IPC import exported by this (the client) process."""

from __future__ import annotations

import uuid
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _plan(rows, steps, position, generation_base=1, import_required=False, token=7, blocks=None):
    from cruise_b200.contract import CONTRACT_VERSION, ResidentEpochPlan, ResidentEpochRequest

    reqs = tuple(
        ResidentEpochRequest(req_id=f"r{row}", row=row, generation=generation_base + row, token_id=token + row,
                             position=position, sequence_length=position + 1, eos_token_id=4095,
                             scheduler_block_ids=((blocks or {}).get(row, row),),
                             device_block_ids=(2 * row, 2 * row + 1), kv_import_required=import_required)
        for row in rows)
    mask = tuple(1 if r in rows else 0 for r in range(4))
    return ResidentEpochPlan(version=CONTRACT_VERSION, graph_batch_size=4, max_steps=steps, logical_capacity=32,
                             requests=reqs, active_mask=mask)


@pytest.fixture()
def pair(cuda_ok, monkeypatch):
    from cruise_b200.build import build
    from cruise_b200.cuda_backend import CudaEpochEngine
    from cruise_b200.sidecar_backend import SidecarEpochEngine

    build()
    path = Path("/dev/shm") / f"cruise-sidecar-{uuid.uuid4().hex[:8]}"
    monkeypatch.setenv("VLLM_ASCEND_RESIDENT_EPOCH_SOCKET", str(path))
    monkeypatch.setenv("VLLM_ASCEND_RESIDENT_EPOCH_MODEL", "tiny")
    monkeypatch.setenv("VLLM_ASCEND_RESIDENT_EPOCH_EXTERNAL_WEIGHTS", "synthetic:0")
    sidecar = SidecarEpochEngine()
    local = CudaEpochEngine(model="tiny", weights="synthetic:0")
    yield sidecar, local
    local.close()
    sidecar.close()
    assert sidecar.process.returncode == 0   # orderly shutdown
    assert not path.exists()


def _same(a, b):
    assert (a.status, a.model_calls, a.token_ids, a.row_generations) == (
        b.status, b.model_calls, b.token_ids, b.row_generations)
    assert a.commit_state == b.commit_state and a.feed_calls == b.feed_calls == 1
    assert (a.kv_imported, a.kv_import_checksum) == (b.kv_imported, b.kv_import_checksum)


def test_warmup_and_epochs(pair):
    sidecar, local = pair
    w = sidecar.warm_up()
    assert (w.status, w.model_calls) == (0, 1) and local.warm_up().model_calls == 1
    first = _plan([0, 1, 2], steps=2, position=0)
    a, b = sidecar.execute(first), local.execute(first)
    _same(a, b)
    assert a.status == 0 and all(len(t) == 2 for t in a.token_ids.values())
    # continue the same generations
    from cruise_b200.contract import CONTRACT_VERSION, ResidentEpochPlan, ResidentEpochRequest

    reqs = tuple(ResidentEpochRequest(req_id=r.req_id, row=r.row, generation=r.generation,
                                      token_id=a.token_ids[r.req_id][-1], position=2, sequence_length=3,
                                      eos_token_id=4095, scheduler_block_ids=(r.row,),
                                      device_block_ids=(2 * r.row, 2 * r.row + 1)) for r in first.requests)
    second = ResidentEpochPlan(version=CONTRACT_VERSION, graph_batch_size=4, max_steps=4, logical_capacity=32,
                               requests=reqs, active_mask=first.active_mask)
    _same(sidecar.execute(second), local.execute(second))


def test_snapshot_and_device_ipc_imports(pair):
    from cruise_b200.kv_transfer import KVGeometry, ResidentKVSnapshot, capture_kv_device_transfer, kv_payload_checksum

    sidecar, local = pair
    g = KVGeometry.of(local.config)
    rows, blocks = (1, 2), {1: 5, 2: 3}
    rng = np.random.default_rng(4)
    values = rng.standard_normal(g.payload_bytes // 2).astype(np.float32) * 0.5
    raw = torch.from_numpy(values).to(torch.bfloat16).view(torch.int16).numpy().reshape(2, g.layers, 4, -1)
    raw[:, :, [0, 3]] = 0
    payload = raw.tobytes()
    mask, gens = 0b0110, (0, 2, 3, 0)
    snapshot = ResidentKVSnapshot(21, mask, gens, payload, kv_payload_checksum(payload, mask, g), g)
    plan = _plan(rows, steps=2, position=3, import_required=True, blocks=blocks)
    a, b = sidecar.execute_with_import(plan, snapshot), local.execute_with_import(plan, snapshot)
    _same(a, b)
    assert a.kv_import_checksum == snapshot.checksum and a.kv_transfer_mode == "host_snapshot"

    # the same blocks exported from this process's memory, imported by the server
    kv = torch.zeros((g.layers, 2, 8, g.block_size, g.kv_heads, g.head_size), dtype=torch.bfloat16, device="cuda:0")
    view = torch.frombuffer(bytearray(payload), dtype=torch.bfloat16).view(
        2, g.layers, 4, g.block_size, g.kv_heads, g.head_size)
    for row, block in blocks.items():
        for layer in range(g.layers):
            for kvi in range(2):
                kv[layer, kvi, block] = view[kvi, layer, row].to("cuda:0")
    torch.cuda.synchronize()
    worker = SimpleNamespace(model_runner=SimpleNamespace(kv_caches=[kv[layer] for layer in range(g.layers)]))
    ipc_plan = _plan(rows, steps=2, position=3, generation_base=11, import_required=True, blocks=blocks)
    transfer = capture_kv_device_transfer(worker, ipc_plan, g)
    c = sidecar.execute_with_device_transfer(ipc_plan, transfer)
    ipc_snapshot = ResidentKVSnapshot(22, mask, (0, 12, 13, 0), payload, kv_payload_checksum(payload, mask, g), g)
    d = local.execute_with_import(ipc_plan, ipc_snapshot)
    assert c.kv_transfer_mode == "device_ipc" and c.kv_import_checksum == ipc_snapshot.checksum
    assert (c.status, c.token_ids, c.row_generations) == (d.status, d.token_ids, d.row_generations)
