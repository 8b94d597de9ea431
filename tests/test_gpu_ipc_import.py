"""Device-IPC KV import across processes (one GPU, two processes).

An exporter process holds a stock-layout paged KV cache (one allocation, the
layers' K/V views in it) with the prompts' blocks filled, and captures the
transfer exactly as a vLLM worker would (``capture_kv_device_transfer``:
``cudaIpcGetMemHandle`` of the allocation + per-layer offsets).  The engine
process imports it through the reference-compatible bridge
(``resident_epoch_execute`` with IPC metadata), which opens the handles and
gathers the blocks with device copies.  The same blocks imported through the
host snapshot on a fresh engine must give the same checksum proof, tokens,
generations and model calls: the two transfer modes carry one payload.
"""

from __future__ import annotations

import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

ROWS = (1, 2)
SOURCE_BLOCKS = {1: 5, 2: 3}   # scheduler block of each importing row in the stock cache


def _plan(position=3, steps=2):
    from cruise_b200.contract import CONTRACT_VERSION, ResidentEpochPlan, ResidentEpochRequest

    reqs = tuple(
        ResidentEpochRequest(req_id=f"r{row}", row=row, generation=1 + row, token_id=7 + row, position=position,
                             sequence_length=position + 1, eos_token_id=4095,
                             scheduler_block_ids=(SOURCE_BLOCKS[row],), device_block_ids=(2 * row, 2 * row + 1),
                             kv_import_required=True)
        for row in ROWS)
    mask = tuple(1 if r in ROWS else 0 for r in range(4))
    return ResidentEpochPlan(version=CONTRACT_VERSION, graph_batch_size=4, max_steps=steps, logical_capacity=32,
                             requests=reqs, active_mask=mask)


def _payload(geometry) -> bytes:
    """Seeded bf16 K/V blocks for the importing rows, zero for the others, in
    the snapshot order [K|V][layer][row][block]."""
    rng = np.random.default_rng(3)
    values = rng.standard_normal(geometry.payload_bytes // 2).astype(np.float32) * 0.5
    raw = torch.from_numpy(values).to(torch.bfloat16).view(torch.int16).numpy().reshape(2, geometry.layers, 4, -1)
    for r in range(4):
        if r not in ROWS:
            raw[:, :, r] = 0
    return raw.tobytes()


def _exporter(queue, done, payload: bytes, geometry_fields: tuple, source_blocks: int) -> None:
    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root))
    sys.path.insert(0, str(root / "tests"))
    import torch

    from cruise_b200.kv_transfer import KVGeometry, capture_kv_device_transfer

    g = KVGeometry(*geometry_fields)
    # the stock cache: [layer][K|V][block][slot][kv head][dim] in one allocation
    kv = torch.zeros((g.layers, 2, source_blocks, g.block_size, g.kv_heads, g.head_size),
                     dtype=torch.bfloat16, device="cuda:0")
    raw = torch.frombuffer(bytearray(payload), dtype=torch.bfloat16).view(
        2, g.layers, 4, g.block_size, g.kv_heads, g.head_size)
    for row, block in SOURCE_BLOCKS.items():
        for layer in range(g.layers):
            for kvi in range(2):
                kv[layer, kvi, block] = raw[kvi, layer, row].to("cuda:0")
    torch.cuda.synchronize()
    worker = SimpleNamespace(model_runner=SimpleNamespace(kv_caches=[kv[layer] for layer in range(g.layers)]))
    queue.put(capture_kv_device_transfer(worker, _plan(), g))
    done.wait(timeout=600)   # the allocation must outlive the importer's copies


def test_device_ipc_import_matches_host_snapshot(cuda_ok):
    from cruise_b200.backend import ResidentEpochBackend
    from cruise_b200.contract import get_result
    from cruise_b200.cuda_backend import CudaEpochEngine
    from cruise_b200.kv_transfer import KVGeometry, ResidentKVSnapshot, kv_payload_checksum

    plan = _plan()
    engine = CudaEpochEngine(model="tiny", weights="synthetic:0")
    g = KVGeometry.of(engine.config)
    payload = _payload(g)
    mask = sum(1 << r for r in ROWS)
    gens = tuple(1 + r if r in ROWS else 0 for r in range(4))
    snapshot = ResidentKVSnapshot(11, mask, gens, payload, kv_payload_checksum(payload, mask, g), g)
    host_out = ResidentEpochBackend(engine).execute(plan, snapshot=snapshot)
    host = get_result(host_out)
    engine.close()
    assert host.kv_imported and host.kv_transfer_mode == "host_snapshot"

    ctx = mp.get_context("spawn")
    queue, done = ctx.Queue(), ctx.Event()
    proc = ctx.Process(target=_exporter, args=(queue, done, payload,
                                               (g.layers, g.block_size, g.kv_heads, g.head_size), 8))
    proc.start()
    try:
        transfer = queue.get(timeout=300)
        assert transfer.import_mask == mask and transfer.row_generations == gens
        engine = CudaEpochEngine(model="tiny", weights="synthetic:0")
        device_out = ResidentEpochBackend(engine).execute(plan, device_transfer=transfer)
        device = get_result(device_out)
        engine.close()
    finally:
        done.set()
        proc.join(timeout=120)
    assert proc.exitcode == 0
    assert device.kv_imported and device.kv_transfer_mode == "device_ipc"
    assert device.kv_import_checksum == host.kv_import_checksum == snapshot.checksum
    assert device_out.sampled_token_ids == host_out.sampled_token_ids
    assert len(host_out.sampled_token_ids) == len(ROWS) and all(len(t) == 2 for t in host_out.sampled_token_ids)
    assert device.model_calls == host.model_calls == 2 and device.computed_steps == host.computed_steps
    assert device.row_generations == host.row_generations
