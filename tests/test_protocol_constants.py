"""Native header constants equal the Python ones (reference tests/test_productization_m0.py:444-473),
and the byte ledger of the epoch ABI (reference tests/test_abi_measurement.py)."""

import re
from pathlib import Path

from cruise_b200 import abi, kv_transfer, version
from cruise_b200.contract import EpochCommitState

ROOT = Path(__file__).resolve().parents[1]


def header_defines() -> dict[str, int]:
    text = (ROOT / "include" / "cruise_protocol.h").read_text()
    return {m.group(1): int(m.group(2), 0) for m in re.finditer(r"#define (\w+) (0x[0-9A-Fa-f]+|\d+)", text)}


def test_protocol_header_matches_python_constants():
    d = header_defines()
    assert d["CRUISE_SIDECAR_PROTOCOL_VERSION"] == version.SIDECAR_PROTOCOL_VERSION
    assert d["CRUISE_SIDECAR_REQUEST_BYTES"] == version.SIDECAR_REQUEST_BYTES
    assert d["CRUISE_SIDECAR_RESPONSE_BYTES"] == version.SIDECAR_RESPONSE_BYTES
    assert d["CRUISE_EPOCH_PREPARED"] == EpochCommitState.PREPARED
    assert d["CRUISE_EPOCH_EXECUTING"] == EpochCommitState.EXECUTING
    assert d["CRUISE_EPOCH_COMMITTED"] == EpochCommitState.COMMITTED
    assert d["CRUISE_RESIDENT_IMPORT_PAYLOAD_BYTES"] == kv_transfer.PAYLOAD_BYTES
    assert d["CRUISE_RESIDENT_TRANSFER_HEADER_BYTES"] == kv_transfer.TRANSFER_HEADER_BYTES
    assert d["CRUISE_RESIDENT_TRANSFER_MAGIC"] == kv_transfer.TRANSFER_MAGIC
    assert d["CRUISE_RESIDENT_IPC_METADATA_MAGIC"] == kv_transfer.IPC_METADATA_MAGIC
    assert d["CRUISE_RESIDENT_IPC_METADATA_HEADER_BYTES"] + 56 * 64 == kv_transfer.IPC_METADATA_BYTES


def test_epoch_abi_byte_ledger():
    assert abi.ABI_BYTES["new"] == {"input": 260, "output": 368}
    assert abi.ABI_BYTES["old"] == {"input": 58_720_516, "output": 78_184_928}
    assert abi.NEW_TOTAL_BYTES == 628 and abi.TOTAL_REDUCTION_BYTES == 136_904_816


def test_bridge_commit_state_transitions_bracket_submission():
    source = (ROOT / "cruise_b200" / "csrc" / "engine.cu").read_text()
    body = source[source.index("int32_t resident_epoch_execute("):]
    prepared = body.index("*output_commit_state = CRUISE_EPOCH_PREPARED")
    executing = body.index("*output_commit_state = CRUISE_EPOCH_EXECUTING")
    submit = body.index("run_epoch(", executing)
    committed = body.index("*output_commit_state = CRUISE_EPOCH_COMMITTED")
    final_return = body.index("return 0;", committed)
    assert prepared < executing < submit < committed < final_return
