"""KV transfer formats (reference tests/test_kv_transfer.py:35-303)."""

import struct
import zlib
from types import SimpleNamespace

import pytest
import torch

from cruise_b200.contract import CONTRACT_VERSION, ResidentEpochPlan, ResidentEpochRequest
import cruise_b200.kv_transfer as kvt
from cruise_b200.kv_transfer import (
    BLOCK_ELEMENTS, ELEMENT_BYTES, GRAPH_BATCH_SIZE, HEADER, IPC_KEY_BYTES, IPC_KEY_COUNT, IPC_METADATA_BYTES,
    IPC_METADATA_HEADER, PAYLOAD_BYTES, TRANSFER_HEADER_BYTES, DeviceKVTransfer, KVGeometry, capture_kv_snapshot,
    kv_payload_checksum, read_kv_snapshot, write_kv_snapshot,
)


def request(row, block, generation=7, position=3):
    return ResidentEpochRequest(req_id=f"r{row}", row=row, generation=generation, token_id=42, position=position,
                                sequence_length=position + 1, eos_token_id=151645, scheduler_block_ids=(block,),
                                device_block_ids=(2 * row, 2 * row + 1), state_owner="host", kv_import_required=True)


def plan_of(*requests, steps=2):
    mask = [0] * 4
    for r in requests:
        mask[r.row] = 1
    return ResidentEpochPlan(version=CONTRACT_VERSION, graph_batch_size=4, max_steps=steps, logical_capacity=256,
                             requests=tuple(requests), active_mask=tuple(mask))


def test_constants_match_the_reference_wire_sizes():
    assert PAYLOAD_BYTES == 29_360_128
    assert HEADER.size == TRANSFER_HEADER_BYTES == 80
    assert IPC_KEY_COUNT == 56 and IPC_METADATA_BYTES == 4088


def test_device_kv_transfer_wire_contract_contains_only_metadata():
    transfer = DeviceKVTransfer(
        transfer_id=7, import_mask=0b0101, row_generations=(11, 0, 13, 0), block_ids=(2, 0, 5, 0),
        source_bytes=8 * BLOCK_ELEMENTS * ELEMENT_BYTES,
        source_offsets=(0, BLOCK_ELEMENTS * ELEMENT_BYTES) * (IPC_KEY_COUNT // 2),
        keys=tuple(bytes([i]) * IPC_KEY_BYTES for i in range(IPC_KEY_COUNT)),
    )
    wire = transfer.wire_bytes()
    assert len(wire) == IPC_METADATA_BYTES
    assert IPC_METADATA_BYTES < PAYLOAD_BYTES // 1000
    assert IPC_METADATA_HEADER.unpack_from(wire)[12:] == transfer.source_offsets
    assert wire[-IPC_KEY_BYTES:] == bytes([IPC_KEY_COUNT - 1]) * IPC_KEY_BYTES
    with pytest.raises(ValueError, match="outside its exported allocation"):
        DeviceKVTransfer(**{**transfer.__dict__, "block_ids": (8, 0, 5, 0)}).validate()


def test_capture_stock_paged_kv_uses_scheduler_block_and_resident_row():
    key = torch.zeros((2, 128, 4, 128), dtype=torch.bfloat16)
    value = torch.zeros_like(key)
    key[1].fill_(1)
    value[1].fill_(2)
    worker = SimpleNamespace(model_runner=SimpleNamespace(kv_caches=[(key, value)] * 28))
    snapshot = capture_kv_snapshot(worker, plan_of(request(1, 1)))
    assert len(snapshot.payload) == PAYLOAD_BYTES
    assert snapshot.import_mask == 0b0010 and snapshot.row_generations == (0, 7, 0, 0)
    assert snapshot.checksum == kv_payload_checksum(snapshot.payload, 0b0010)
    row_bytes = BLOCK_ELEMENTS * ELEMENT_BYTES
    value_base = 28 * GRAPH_BATCH_SIZE * row_bytes
    assert struct.unpack_from("<H", snapshot.payload, row_bytes)[0] == 0x3F80          # 1.0 in bf16
    assert struct.unpack_from("<H", snapshot.payload, value_base + row_bytes)[0] == 0x4000   # 2.0
    assert struct.unpack_from("<H", snapshot.payload, 0)[0] == 0


def test_capture_stock_paged_kv_imports_multiple_scheduler_blocks_by_row():
    key = torch.zeros((4, 128, 4, 128), dtype=torch.bfloat16)
    value = torch.zeros_like(key)
    for block in range(4):
        key[block].fill_(block + 1)
        value[block].fill_(block + 5)
    worker = SimpleNamespace(model_runner=SimpleNamespace(kv_caches=[(key, value)] * 28))
    snapshot = capture_kv_snapshot(worker, plan_of(request(0, 2), request(2, 0), request(3, 3), steps=1))
    assert snapshot.import_mask == 0b1101
    row_bytes = BLOCK_ELEMENTS * ELEMENT_BYTES
    for row, word in {0: 0x4040, 1: 0, 2: 0x3F80, 3: 0x4080}.items():
        assert struct.unpack_from("<H", snapshot.payload, row * row_bytes)[0] == word


def test_stacked_kv_layout_is_accepted():
    cache = torch.zeros((2, 3, 128, 4, 128), dtype=torch.bfloat16)
    cache[0, 2].fill_(1)
    worker = SimpleNamespace(model_runner=SimpleNamespace(kv_caches=[cache] * 28))
    snapshot = capture_kv_snapshot(worker, plan_of(request(0, 2)))
    assert struct.unpack_from("<H", snapshot.payload, 0)[0] == 0x3F80


def test_checksum_is_zlib_adler_chained_over_imported_blocks():
    g = KVGeometry(layers=2, block_size=16, kv_heads=2, head_size=64)
    payload = bytes((i * 7 + 3) & 0xFF for i in range(g.payload_bytes))
    expected = 1
    half = g.payload_bytes // 2
    for cache in range(2):
        for layer in range(2):
            for row in (0, 3):
                start = cache * half + (layer * 4 + row) * g.block_bytes
                expected = zlib.adler32(payload[start:start + g.block_bytes], expected)
    assert kv_payload_checksum(payload, 0b1001, g) == expected


def test_snapshot_file_round_trip(tmp_path):
    g = KVGeometry(layers=2, block_size=16, kv_heads=2, head_size=64)
    payload = bytes(range(256)) * (g.payload_bytes // 256)
    snapshot = kvt.ResidentKVSnapshot(5, 0b0011, (3, 4, 0, 0), payload, kv_payload_checksum(payload, 3, g), g)
    path = f"/dev/shm/cruise-test-{id(snapshot)}"
    try:
        write_kv_snapshot(path, snapshot)
        back = read_kv_snapshot(path, g)
        assert back.checksum == snapshot.checksum and back.payload == payload and back.row_generations == (3, 4, 0, 0)
    finally:
        import os
        if os.path.exists(path):
            os.unlink(path)
    with pytest.raises(ValueError, match="/dev/shm"):
        write_kv_snapshot(tmp_path / "x", snapshot)


def test_device_transfer_capture_uses_allocation_base_offsets(monkeypatch):
    class FakeTensor:
        def __init__(self, ptr):
            self.ptr = ptr

        def is_contiguous(self):
            return True

        def data_ptr(self):
            return self.ptr

    view_bytes = 8 * BLOCK_ELEMENTS * ELEMENT_BYTES
    caches = []
    for layer in range(28):
        base = 0x10_0000_0000 + layer * 0x1000_0000
        caches.append((FakeTensor(base), FakeTensor(base + view_bytes)))
    monkeypatch.setattr(kvt, "_allocation_range", lambda ptr: (ptr - ptr % 0x1000_0000, 4 * view_bytes))
    monkeypatch.setattr(kvt, "_ipc_handle", lambda base: base.to_bytes(8, "little") * 8)
    worker = SimpleNamespace(model_runner=SimpleNamespace(kv_caches=caches))
    transfer = kvt.capture_kv_device_transfer(worker, plan_of(request(0, 3)))
    assert transfer.source_offsets == (0, view_bytes) * 28
    assert transfer.keys[0] == transfer.keys[1] and len(transfer.keys[0]) == IPC_KEY_BYTES
    assert len(transfer.wire_bytes()) == IPC_METADATA_BYTES
