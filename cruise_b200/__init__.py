"""cruise_b200 -- B200-native resident decode-epoch engine.

The hot path (a whole K-step greedy decode epoch of a Qwen2-architecture
model over a paged KV cache) runs as one persistent sm_100a kernel in
``libcruise_epoch.so``; this package holds the host-side mirror of the
reference's operator surface (epoch contract, backend, KV transfer) and the
ctypes binding of the engine's C ABI.
"""

from .model_config import BATCH, MAX_STEPS, PRESETS, QWEN25_7B, TINY, ModelConfig

__all__ = ["BATCH", "MAX_STEPS", "PRESETS", "QWEN25_7B", "TINY", "ModelConfig"]
