"""krystal_b200 — a B200-native backend for Krystal's batched frame forward.

Host side of the drop-in boundary: the C ABI (include/krystal_cuda.h,
krystal_b200/_lib/libkrystal_cuda.so) bound through ctypes, plus the host
logic the reference keeps on the host (frame packing, weight init, the
selection mask). The CUDA library is required: constructing a backend raises
when it is missing; nothing falls back to the CPU.
"""
from .frame import (FrameBatch, HostFrame, HostFrameError, HostRecord, HostToken, PAD_TOKEN, QUERY_BAND,
                    compile_active_frame, pack_frame_batch, pack_host_frame, record_ranges)
from .model import (BRAIN_FORWARD_CONFIG, RECORD_WIDTH, BrainForwardConfig, BrainForwardWeights,
                    create_brain_forward_weights, embedding_table_bases, weight_layout)

__all__ = [
    "FrameBatch", "HostFrame", "HostFrameError", "HostRecord", "HostToken", "PAD_TOKEN", "QUERY_BAND",
    "RECORD_WIDTH", "compile_active_frame", "pack_frame_batch", "pack_host_frame", "record_ranges",
    "BRAIN_FORWARD_CONFIG", "BrainForwardConfig", "BrainForwardWeights", "create_brain_forward_weights",
    "embedding_table_bases", "weight_layout", "cuda_backend", "CudaBrainBackend", "BrainSession",
]


def __getattr__(name):
    if name in ("cuda_backend", "CudaBrainBackend"):
        from . import backend
        return getattr(backend, name)
    if name == "BrainSession":
        from .session import BrainSession
        return BrainSession
    raise AttributeError(name)
