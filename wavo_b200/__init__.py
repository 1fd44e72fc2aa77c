"""wavo_b200: a B200-native (sm_100a) CUDA implementation of the multi-head attention path of
vladkens/wavo — the encoders' self-attention with its projections and the Whisper decoder's
attention over F16 KV caches — behind a C ABI (include/wavo_cuda.h) that mirrors the reference's
GPU backend op interface (src/gpu/mod.rs `Gpu` / `Pass`).

`wavo_b200.gpu` is the host-side mirror of that interface; `wavo_b200.runner` shards independent
segments over the GPUs of one node.
"""

from ._lib import EPILOGUES, GGML_BF16, GGML_F16, GGML_F32, GGML_Q8_0, WavoError  # noqa: F401

__all__ = ["EPILOGUES", "GGML_BF16", "GGML_F16", "GGML_F32", "GGML_Q8_0", "WavoError"]
