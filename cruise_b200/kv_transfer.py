"""One-shot host-to-device Paged-KV ownership import.

Restates ``src/vllm_ascend_resident_epoch/kv_transfer.py``:

* the snapshot payload (``:362-428``): ``[K|V][layers][4 rows][block][kv_heads][head_dim]``
  bf16 holding each imported row's first scheduler block, zero for other rows;
* its checksum (``:159-174``): zlib Adler-32 chained over K then V, layer-major,
  row-minor, imported rows only (the engine recomputes it on the device over
  the blocks it wrote, ``controller/g4c_b4_resident_epoch.cpp:419-432``);
* the 80-byte transfer-file header (``:23,431-466``) read by the bridge;
* the device-IPC metadata (``:68-137``, 4,088 bytes): 56 keys of 64 bytes.  On
  CUDA a key is the raw ``cudaIpcMemHandle_t`` of the exporting process's K or
  V allocation, and ``source_offsets`` locate each layer's cache inside it.

Geometry defaults are the 7B preset (28 layers, block 128, 4 KV heads of 128);
every function also takes an explicit :class:`KVGeometry`.
"""

from __future__ import annotations

import os
import secrets
import struct
import zlib
from dataclasses import dataclass
from pathlib import Path
from typing import Any

TRANSFER_MAGIC = 0x4352554953454B56  # "CRUISEKV"
TRANSFER_VERSION = 1
TRANSFER_HEADER_BYTES = 80
IPC_METADATA_MAGIC = 0x4352554953454950  # "CRUISEIP"
IPC_METADATA_VERSION = 2
IPC_KEY_BYTES = 64
GRAPH_BATCH_SIZE = 4
HEADER = struct.Struct("<QIIQQI4i7I")


@dataclass(frozen=True)
class KVGeometry:
    layers: int = 28
    block_size: int = 128
    kv_heads: int = 4
    head_size: int = 128
    element_bytes: int = 2

    @property
    def block_elements(self) -> int:
        return self.block_size * self.kv_heads * self.head_size

    @property
    def block_bytes(self) -> int:
        return self.block_elements * self.element_bytes

    @property
    def payload_bytes(self) -> int:
        return 2 * self.layers * GRAPH_BATCH_SIZE * self.block_bytes

    @property
    def ipc_keys(self) -> int:
        return 2 * self.layers

    @classmethod
    def of(cls, config: Any) -> "KVGeometry":
        """Geometry of a :class:`cruise_b200.model_config.ModelConfig`."""
        return cls(config.num_layers, config.block_size, config.num_kv_heads, config.head_dim)


DEFAULT_GEOMETRY = KVGeometry()
LAYERS = DEFAULT_GEOMETRY.layers
BLOCK_SIZE = DEFAULT_GEOMETRY.block_size
NUM_KV_HEADS = DEFAULT_GEOMETRY.kv_heads
HEAD_SIZE = DEFAULT_GEOMETRY.head_size
ELEMENT_BYTES = DEFAULT_GEOMETRY.element_bytes
BLOCK_ELEMENTS = DEFAULT_GEOMETRY.block_elements
PAYLOAD_BYTES = DEFAULT_GEOMETRY.payload_bytes          # 29,360,128
IPC_KEY_COUNT = DEFAULT_GEOMETRY.ipc_keys               # 56
IPC_METADATA_HEADER = struct.Struct(f"<QIIQ4i4i{IPC_KEY_COUNT}Q")
IPC_METADATA_BYTES = IPC_METADATA_HEADER.size + IPC_KEY_COUNT * IPC_KEY_BYTES   # 4,088


def kv_payload_checksum(payload: bytes, import_mask: int, geometry: KVGeometry = DEFAULT_GEOMETRY) -> int:
    """Adler-32 over the imported rows' blocks: K then V, layer-major, row-minor."""
    if len(payload) != geometry.payload_bytes:
        raise ValueError("cannot checksum an incomplete KV transfer payload")
    view = memoryview(payload)
    cache_bytes = geometry.payload_bytes // 2
    checksum = 1
    for cache in range(2):
        for layer in range(geometry.layers):
            for row in range(GRAPH_BATCH_SIZE):
                if import_mask & (1 << row):
                    start = cache * cache_bytes + (layer * GRAPH_BATCH_SIZE + row) * geometry.block_bytes
                    checksum = zlib.adler32(view[start : start + geometry.block_bytes], checksum)
    return checksum & 0xFFFFFFFF


@dataclass(frozen=True)
class ResidentKVSnapshot:
    transfer_id: int
    import_mask: int
    row_generations: tuple[int, ...]
    payload: bytes
    checksum: int
    geometry: KVGeometry = DEFAULT_GEOMETRY

    def validate(self) -> None:
        if self.transfer_id <= 0:
            raise ValueError("KV transfer id must be positive")
        if len(self.row_generations) != GRAPH_BATCH_SIZE:
            raise ValueError("KV transfer generation vector must have four rows")
        if any(g < 0 for g in self.row_generations):
            raise ValueError("KV transfer generations must be non-negative")
        if not 0 < self.import_mask < 1 << GRAPH_BATCH_SIZE:
            raise ValueError("KV transfer mask must select at least one row")
        for row, generation in enumerate(self.row_generations):
            if bool(self.import_mask & (1 << row)) != (generation > 0):
                raise ValueError("KV transfer mask and generations disagree")
        if len(self.payload) != self.geometry.payload_bytes:
            raise ValueError(
                f"KV transfer payload must be {self.geometry.payload_bytes} bytes, got {len(self.payload)}"
            )
        if self.checksum != kv_payload_checksum(self.payload, self.import_mask, self.geometry):
            raise ValueError("KV transfer checksum does not match its payload")

    def header_bytes(self) -> bytes:
        g = self.geometry
        return HEADER.pack(
            TRANSFER_MAGIC, TRANSFER_VERSION, TRANSFER_HEADER_BYTES, self.transfer_id, len(self.payload),
            self.import_mask, *self.row_generations, g.layers, GRAPH_BATCH_SIZE, g.block_size, g.kv_heads,
            g.head_size, g.element_bytes, self.checksum,
        )


@dataclass(frozen=True)
class DeviceKVTransfer:
    """Metadata for importing stock KV blocks device to device (no host payload)."""

    transfer_id: int
    import_mask: int
    row_generations: tuple[int, ...]
    block_ids: tuple[int, ...]
    source_bytes: int
    source_offsets: tuple[int, ...]
    keys: tuple[bytes, ...]
    geometry: KVGeometry = DEFAULT_GEOMETRY

    def validate(self) -> None:
        g = self.geometry
        if self.transfer_id <= 0:
            raise ValueError("device KV transfer id must be positive")
        if len(self.row_generations) != GRAPH_BATCH_SIZE:
            raise ValueError("device KV transfer generation vector must have four rows")
        if len(self.block_ids) != GRAPH_BATCH_SIZE:
            raise ValueError("device KV transfer block vector must have four rows")
        if not 0 < self.import_mask < 1 << GRAPH_BATCH_SIZE:
            raise ValueError("device KV transfer mask must select at least one row")
        if self.source_bytes <= 0:
            raise ValueError("device KV transfer source size must be positive")
        if len(self.source_offsets) != IPC_KEY_COUNT or len(self.keys) != IPC_KEY_COUNT:
            raise ValueError(f"device KV transfer must carry {IPC_KEY_COUNT} keys and source offsets")
        for row in range(GRAPH_BATCH_SIZE):
            selected = bool(self.import_mask & (1 << row))
            generation, block = self.row_generations[row], self.block_ids[row]
            if selected:
                if generation <= 0 or block < 0:
                    raise ValueError("selected device KV rows need generation and block")
                for offset in self.source_offsets[: g.ipc_keys]:
                    if offset < 0 or offset + (block + 1) * g.block_bytes > self.source_bytes:
                        raise ValueError("device KV block is outside its exported allocation")
            elif generation != 0 or block != 0:
                raise ValueError("unselected device KV rows must be zeroed")
        for key in self.keys:
            if not key or len(key) > IPC_KEY_BYTES:
                raise ValueError("device KV IPC key does not fit the wire contract")

    def wire_bytes(self) -> bytes:
        self.validate()
        header = IPC_METADATA_HEADER.pack(
            IPC_METADATA_MAGIC, IPC_METADATA_VERSION, self.import_mask, self.source_bytes,
            *self.row_generations, *self.block_ids, *self.source_offsets,
        )
        payload = header + b"".join(key.ljust(IPC_KEY_BYTES, b"\0") for key in self.keys)
        if len(payload) != IPC_METADATA_BYTES:
            raise AssertionError("device KV IPC metadata ABI size changed")
        return payload


def _layer_pair(layer_cache: Any):
    """(key, value) of one layer of a stock vLLM cache: a (K, V) pair or a
    tensor whose leading dimension of 2 holds K and V."""
    if isinstance(layer_cache, (tuple, list)) and len(layer_cache) >= 2:
        return layer_cache[0], layer_cache[1]
    shape = getattr(layer_cache, "shape", None)
    if shape is not None and len(shape) >= 1 and shape[0] == 2:
        return layer_cache[0], layer_cache[1]
    raise RuntimeError("stock vLLM KV cache layer is not a K/V pair")


def capture_kv_snapshot(worker: Any, plan: Any, geometry: KVGeometry = DEFAULT_GEOMETRY) -> ResidentKVSnapshot:
    """Copies each importing row's first scheduler block out of the stock vLLM
    KV cache (``worker.model_runner.kv_caches``) into a snapshot."""
    import torch

    requests = [r for r in plan.requests if r.kv_import_required]
    if not requests:
        raise ValueError("KV snapshot requested for a plan without imports")
    if plan.logical_capacity > geometry.block_size * 2:
        raise ValueError("an import covers at most the rows' two blocks")
    caches = getattr(getattr(worker, "model_runner", None), "kv_caches", None)
    if not isinstance(caches, list) or len(caches) != geometry.layers:
        raise RuntimeError("stock vLLM KV cache layout does not match the engine's layers")
    by_row = {r.row: r for r in requests}
    block_shape = (geometry.block_size, geometry.kv_heads, geometry.head_size)
    payload = torch.zeros((2, geometry.layers, GRAPH_BATCH_SIZE) + block_shape, dtype=torch.bfloat16)
    for layer, layer_cache in enumerate(caches):
        key, value = _layer_pair(layer_cache)
        for row, request in by_row.items():
            if len(request.scheduler_block_ids) != 1:
                raise ValueError("the import takes one scheduler block per row")
            block = request.scheduler_block_ids[0]
            if not 0 <= block < key.shape[0]:
                raise ValueError("scheduler block is outside the stock KV cache")
            if tuple(key[block].shape) != block_shape or tuple(value[block].shape) != block_shape:
                raise RuntimeError("stock vLLM KV block shape differs from the engine layout")
            payload[0, layer, row] = key[block].detach().to("cpu", torch.bfloat16)
            payload[1, layer, row] = value[block].detach().to("cpu", torch.bfloat16)
    raw = payload.contiguous().view(torch.int16).numpy().tobytes()
    mask = sum(1 << r.row for r in requests)
    generations = [0] * GRAPH_BATCH_SIZE
    for r in requests:
        generations[r.row] = r.generation
    snapshot = ResidentKVSnapshot(
        transfer_id=secrets.randbits(63) or 1, import_mask=mask, row_generations=tuple(generations),
        payload=raw, checksum=kv_payload_checksum(raw, mask, geometry), geometry=geometry,
    )
    snapshot.validate()
    return snapshot


def write_kv_snapshot(path: str | Path, snapshot: ResidentKVSnapshot) -> None:
    """Atomically writes header + payload to a file under /dev/shm."""
    snapshot.validate()
    destination = Path(path).resolve()
    if not str(destination).startswith("/dev/shm/"):
        raise ValueError("KV transfer files must be under /dev/shm")
    destination.parent.mkdir(parents=True, exist_ok=True)
    temporary = destination.with_name(f".{destination.name}.tmp-{os.getpid()}-{snapshot.transfer_id}")
    if temporary.exists():
        raise RuntimeError(f"stale KV transfer temporary file exists: {temporary}")
    try:
        with temporary.open("xb") as stream:
            stream.write(snapshot.header_bytes())
            stream.write(snapshot.payload)
            stream.flush()
            os.fsync(stream.fileno())
        os.replace(temporary, destination)
    finally:
        temporary.unlink(missing_ok=True)


def read_kv_snapshot(path: str | Path, geometry: KVGeometry = DEFAULT_GEOMETRY) -> ResidentKVSnapshot:
    data = Path(path).read_bytes()
    fields = HEADER.unpack_from(data)
    magic, version, header_bytes, transfer_id, payload_bytes, mask = fields[:6]
    generations = tuple(fields[6:10])
    layers, batch, block, heads, head, element, checksum = fields[10:]
    if (magic, version, header_bytes) != (TRANSFER_MAGIC, TRANSFER_VERSION, TRANSFER_HEADER_BYTES):
        raise ValueError("not a resident KV transfer file")
    if (layers, batch, block, heads, head, element) != (
        geometry.layers, GRAPH_BATCH_SIZE, geometry.block_size, geometry.kv_heads, geometry.head_size,
        geometry.element_bytes,
    ):
        raise ValueError("KV transfer file geometry differs from the engine's")
    payload = data[TRANSFER_HEADER_BYTES:]
    if len(payload) != payload_bytes:
        raise ValueError("truncated KV transfer file")
    snapshot = ResidentKVSnapshot(transfer_id, mask, generations, payload, checksum, geometry)
    snapshot.validate()
    return snapshot


# ---- device IPC export (CUDA) ------------------------------------------------------
def _cuda_runtime():
    from cuda.bindings import driver, runtime

    return runtime, driver


def _allocation_range(pointer: int) -> tuple[int, int]:
    _, driver = _cuda_runtime()
    err, base, size = driver.cuMemGetAddressRange(pointer)
    if int(err) != 0 or int(base) == 0 or int(size) == 0:
        raise RuntimeError(f"cuMemGetAddressRange failed for the stock KV cache ({err})")
    return int(base), int(size)


def _ipc_handle(pointer: int) -> bytes:
    runtime, _ = _cuda_runtime()
    err, handle = runtime.cudaIpcGetMemHandle(pointer)
    if int(err) != 0:
        raise RuntimeError(f"cudaIpcGetMemHandle failed for the stock KV cache ({err})")
    raw = bytes(handle.reserved)
    if len(raw) != IPC_KEY_BYTES:
        raise RuntimeError("unexpected CUDA IPC handle size")
    return raw


def capture_kv_device_transfer(worker: Any, plan: Any, geometry: KVGeometry = DEFAULT_GEOMETRY) -> DeviceKVTransfer:
    """IPC metadata for importing the stock KV blocks without a host copy:
    one handle per K and V layer allocation plus each layer's offset in it."""
    requests = [r for r in plan.requests if r.kv_import_required]
    if not requests:
        raise ValueError("device KV transfer requested for a plan without imports")
    caches = getattr(getattr(worker, "model_runner", None), "kv_caches", None)
    if not isinstance(caches, list) or len(caches) != geometry.layers:
        raise RuntimeError("stock vLLM KV cache layout does not match the engine's layers")
    keys, offsets, sizes = [], [], set()
    for layer_cache in caches:
        for tensor in _layer_pair(layer_cache):
            if not tensor.is_contiguous():
                raise RuntimeError("stock KV cache entries must be contiguous for IPC export")
            base, size = _allocation_range(int(tensor.data_ptr()))
            keys.append(_ipc_handle(base))
            offsets.append(int(tensor.data_ptr()) - base)
            sizes.add(size)
    if len(sizes) != 1:
        raise RuntimeError("key/value KV allocations do not have a common size")
    block_ids = [0] * GRAPH_BATCH_SIZE
    generations = [0] * GRAPH_BATCH_SIZE
    for r in requests:
        if len(r.scheduler_block_ids) != 1:
            raise ValueError("device KV IPC requires one scheduler block per row")
        block_ids[r.row] = int(r.scheduler_block_ids[0])
        generations[r.row] = int(r.generation)
    keys += [keys[-1]] * (IPC_KEY_COUNT - len(keys))
    offsets += [offsets[-1]] * (IPC_KEY_COUNT - len(offsets))
    transfer = DeviceKVTransfer(
        transfer_id=secrets.randbits(63) or 1, import_mask=sum(1 << r.row for r in requests),
        row_generations=tuple(generations), block_ids=tuple(block_ids), source_bytes=sizes.pop(),
        source_offsets=tuple(offsets), keys=tuple(keys), geometry=geometry,
    )
    transfer.validate()
    return transfer
