"""Versions of the contracts this engine speaks (src/vllm_ascend_resident_epoch/version.py:3-17).

The Python epoch contract, the sidecar wire protocol and the two device ABIs
keep the reference's version numbers so that schedulers, workers and servers
built against the reference interoperate with this engine unchanged.
"""

PACKAGE_VERSION = "0.1.0"
PYTHON_CONTRACT_VERSION = 3
SIDECAR_PROTOCOL_VERSION = 7
SIDECAR_REQUEST_BYTES = 136
SIDECAR_RESPONSE_BYTES = 352
HOST_UDF_ABI_VERSION = 2      # the 8-input / 2-output epoch ABI
HOST_UDF_INPUTS = 8
HOST_UDF_OUTPUTS = 2
DECODER_ABI_VERSION = 1       # the 9-input / 4-output decoder-step ABI
DECODER_INPUTS = 9
DECODER_OUTPUTS = 4
