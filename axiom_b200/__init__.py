"""B200-native (sm_100a) Kimi Delta Attention: chunked forward, fused backward
and recurrent decode behind the C ABI in ``include/kda_b200.h``, and the
per-token work around them (prologue, output gate, fused decode step, packed
sequences) behind ``include/kda_mixer.h``; ``layer`` wires a whole mixer
layer."""

from . import layer, mixer  # noqa: F401
from .kda import (  # noqa: F401
    CHUNK, KDA_CC_IMPLS, TILE, cc_scan, check_device, chunk_kda, chunk_kda_varlen, ckpt_states, decode_step,
    device_available, device_status, kda_bwd, kda_bwd_varlen, kda_cc_impl, kda_fwd, kda_fwd_varlen, kernel,
    kernel_bwd, packing, selftest_wait_timeout,
)

__all__ = [
    "CHUNK", "TILE", "KDA_CC_IMPLS", "cc_scan", "check_device", "chunk_kda", "chunk_kda_varlen", "ckpt_states",
    "decode_step", "device_available", "device_status", "kda_bwd", "kda_bwd_varlen", "kda_cc_impl", "kda_fwd",
    "kda_fwd_varlen", "kernel", "kernel_bwd", "layer", "mixer", "packing", "selftest_wait_timeout",
]
