"""B200-native (sm_100a) Kimi Delta Attention core: chunked forward, fused
backward and recurrent decode, behind the C ABI in ``include/kda_b200.h``."""

from .kda import (  # noqa: F401
    CHUNK, KDA_CC_IMPLS, TILE, cc_scan, chunk_kda, ckpt_states, decode_step, device_available,
    kda_bwd, kda_cc_impl, kda_fwd, kernel, kernel_bwd,
)

__all__ = [
    "CHUNK", "TILE", "KDA_CC_IMPLS", "cc_scan", "chunk_kda", "ckpt_states", "decode_step",
    "device_available",
    "kda_bwd", "kda_cc_impl", "kda_fwd", "kernel", "kernel_bwd",
]
