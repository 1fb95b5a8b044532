"""ctypes binding of the C ABI in include/krystal_cuda.h.

The shared library is the product; this module only declares its structs and
signatures and turns a non-OK status into ``KrystalCudaError`` carrying the
library's message. Loading fails loudly when the library is missing or does
not export a declared symbol: there is no fallback path.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libkrystal_cuda.so"

KC_OK = 0
KC_ERR_INVALID_ARG = 1
KC_ERR_CAPACITY = 2
KC_ERR_CUDA = 3
KC_ERR_TIMEOUT = 4
KC_ERR_NONFINITE = 5
KC_ERR_NO_DEVICE = 6
STATUS_NAMES = {0: "OK", 1: "INVALID_ARG", 2: "CAPACITY", 3: "CUDA", 4: "TIMEOUT", 5: "NONFINITE", 6: "NO_DEVICE"}
KC_NO_SELECTION = 0xFFFFFFFF
KC_PRECISION_EXACT = 0
KC_PRECISION_CERTIFIED = 1
KC_PRECISION_FAST = 2
KC_INJECT_ATTN, KC_INJECT_FFN, KC_INJECT_GEMM, KC_INJECT_EXACT_GEMM = 0, 1, 2, 3  # kc_inject_wait_expiry (test hook)
KC_MAX_BANK = 4096
KC_NO_TARGET = 0xFFFFFFFF
KC_AWAY_TARGET = 0x80000000
KC_LEARN_STATS = 8
KC_NO_WORD = 0xFFFFFFFF
CHECKPOINT_REFUSALS = {1: "not a krystal checkpoint", 2: "a later checkpoint format", 3: "a different geometry",
                       4: "a different vocabulary", 5: "truncated"}

# Every function include/krystal_cuda.h declares.
EXPORTS = ("kc_abi_version", "kc_create", "kc_sync", "kc_encode", "kc_select", "kc_forward_batch",
           "kc_forward_batch_device", "kc_set_stream", "kc_get_stream", "kc_synchronize", "kc_profile",
           "kc_profile_read", "kc_launch_count", "kc_destroy", "kc_last_error", "kc_select_noalloc",
           "kc_set_precision", "kc_backward", "kc_backward_batch_device", "kc_learn_frame_stats",
           "kc_learn_accumulate", "kc_stream_create", "kc_stream_push", "kc_stream_flush", "kc_stream_pending",
           "kc_stream_poll", "kc_stream_clock_ms", "kc_stream_last_error", "kc_stream_destroy",
           "kc_stream_push_many", "kc_load_checkpoint", "kc_save_checkpoint", "kc_select_batch",
           "kc_inject_wait_expiry", "kc_learn_plan", "kc_learn_accumulate_rows", "kc_learn_apply",
           "kc_copy_weights", "kc_stream_create_ex", "kc_stream_read_stats")


class KrystalCudaError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status
        self.message = message


P = C.c_void_p
u32p = C.POINTER(C.c_uint32)
f32p = C.POINTER(C.c_float)


class KcConfig(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in (
        "hidden_size", "head_count", "head_dim", "ffn_size", "encoder_blocks", "mixer_blocks", "token_space",
        "field_space", "schema_space", "band_space", "stream_space", "pos_space", "route_kind_count")] + [
        ("token_rows", P), ("token_rows_len", C.c_uint32)]


class KcBlockView(C.Structure):
    _fields_ = [("wq", P), ("wk", P), ("wv", P), ("w1", P), ("w2", P)]


class KcWeightsView(C.Structure):
    _fields_ = [("embeddings", P), ("enc", C.POINTER(KcBlockView)), ("pool", P), ("mixer", C.POINTER(KcBlockView)),
                ("selector_wq", P), ("selector_wk", P), ("decision_head_wh", P), ("value_head_wv", P)]


class KcChanges(C.Structure):
    _fields_ = [("selector", C.c_int32), ("pool", C.c_int32), ("value_head", C.c_int32),
                ("decision_head", C.c_int32), ("blocks", C.c_int32), ("embedding_rows", P),
                ("embedding_rows_count", C.c_uint32)]


class KcFrameView(C.Structure):
    _fields_ = [("slots", C.c_uint32), ("token_ids", P), ("field_roles", P), ("schema_ids", P), ("band_ids", P),
                ("active_record_indices", P)]


class KcEncodedView(C.Structure):
    _fields_ = [("q", C.c_uint32), ("r", C.c_uint32), ("query_output", P), ("bank_keys", P), ("bank_values", P)]


class KcMaskRule(C.Structure):
    _fields_ = [("schema_allow", P), ("band_allow", P), ("bank_schema_ids", P), ("bank_band_ids", P)]


class KcBatchView(C.Structure):
    _fields_ = [("frames", C.c_uint32), ("records", C.c_uint64), ("rec_off", P), ("token_ids", P),
                ("field_roles", P), ("schema_ids", P), ("band_ids", P), ("schema_allow", P), ("band_allow", P),
                ("uniforms", P), ("word_ids", P), ("word_alpha", C.c_float), ("mask", P)]


class KcBatchOut(C.Structure):
    _fields_ = [("p", P), ("p_capacity", C.c_uint64), ("index", P), ("q_capacity", C.c_uint64), ("p_off", P),
                ("q_off", P), ("query_output", P), ("total_p", C.c_uint64), ("total_q", C.c_uint64),
                ("total_r", C.c_uint64), ("total_t", C.c_uint64)]


class KcBatchSelectView(C.Structure):
    _fields_ = [("schema_allow", P), ("band_allow", P), ("uniforms", P), ("mask", P)]


class KcDeviceResult(C.Structure):
    _fields_ = [("p", P), ("index", P), ("p_off", P), ("q_off", P), ("total_p", C.c_uint64),
                ("total_q", C.c_uint64), ("total_r", C.c_uint64), ("total_t", C.c_uint64)]


class KcBackwardOut(C.Structure):
    _fields_ = [("policy", P), ("value_prediction", P), ("value_loss", C.c_double), ("d_selector_wq", P),
                ("d_selector_wk", P), ("d_pool", P), ("d_field_states", P), ("d_value_wv", P),
                ("p_capacity", C.c_uint64), ("q_capacity", C.c_uint64), ("t_capacity", C.c_uint64),
                ("q", C.c_uint32), ("r", C.c_uint32), ("t", C.c_uint32)]


class KcBackwardResult(C.Structure):
    _fields_ = [("policy", P), ("value_prediction", P), ("value_loss", P), ("d_selector_wq", P),
                ("d_selector_wk", P), ("d_pool", P), ("d_field_states", P), ("d_value_wv", P), ("p_off", P),
                ("q_off", P), ("r_off", P), ("t_off", P), ("total_p", C.c_uint64), ("total_q", C.c_uint64),
                ("total_r", C.c_uint64), ("total_t", C.c_uint64)]


class KcLearnOptions(C.Structure):
    _fields_ = [("learning_rate", C.c_double), ("policy_scale", C.c_double), ("advantage_clip", C.c_double),
                ("max_parameter_abs", C.c_double), ("token_rate", C.c_double), ("unfreeze_pool", C.c_int32),
                ("unfreeze_tokens", C.c_int32)]


KC_LEARN_ROW, KC_LEARN_REPORT, KC_LEARN_RESULT = 10, 9, 19


class KcStreamResult(C.Structure):
    _fields_ = [("first_ticket", C.c_uint64), ("frames", C.c_uint32), ("questions", C.c_uint64),
                ("total_p", C.c_uint64), ("p_off", P), ("q_off", P), ("p", P), ("index", P), ("status", C.c_int),
                ("error", C.c_char_p), ("sealed_ms", C.c_double), ("done_ms", C.c_double),
                ("started_ms", C.c_double), ("sync_wait_ms", C.c_double)]


class KcStreamOptions(C.Structure):
    _fields_ = [("push_threads", C.c_uint32), ("bind_cpus", C.c_int32)]


class KcStreamStats(C.Structure):
    _fields_ = [("batches", C.c_uint64), ("push_calls", C.c_uint64), ("frames_pushed", C.c_uint64),
                ("bytes_staged", C.c_uint64), ("push_ms", C.c_double), ("run_ms", C.c_double),
                ("sync_wait_ms", C.c_double), ("idle_ms", C.c_double), ("workspace_grows", C.c_uint64),
                ("workspace_grow_ms", C.c_double)] + [
        (n, C.c_uint64) for n in ("worker_minor_faults", "worker_major_faults", "worker_voluntary_switches",
                                  "worker_involuntary_switches", "worker_cpu_moves", "caller_minor_faults",
                                  "caller_involuntary_switches")] + [
        (n, C.c_int32) for n in ("gpu_numa_node", "staging_numa_node", "worker_numa_node", "caller_numa_node")] + [
        ("push_threads", C.c_uint32), ("bound_cpus", C.c_uint32)]


class KcStageTimes(C.Structure):
    _fields_ = [(n, C.c_double) for n in ("pack_ms", "embed_ms", "enc_gemm_ms", "enc_attn_ms", "pool_ms",
                                          "mixer_ms", "selector_ms", "total_ms")] + [
        ("enc_gemm_launches", C.c_uint64), ("launches", C.c_uint64), ("batches", C.c_uint64),
        ("enc_gemm_flops", C.c_double), ("fallback_ms", C.c_double), ("fallback_frames", C.c_uint64),
        ("enc_gemm_bytes", C.c_double), ("enc_ffn_ms", C.c_double), ("enc_ffn_launches", C.c_uint64),
        ("enc_ffn_flops", C.c_double), ("enc_ffn_bytes", C.c_double), ("enc_attn_tc_ms", C.c_double),
        ("enc_attn_tc_launches", C.c_uint64), ("enc_attn_tc_flops", C.c_double), ("enc_attn_tc_bytes", C.c_double),
        ("cert_audit_max", C.c_double), ("cert_audit_violations", C.c_uint64), ("cert_audit_frames", C.c_uint64),
        ("cert_kappa0", C.c_double), ("oz_products", C.c_uint64), ("oz_outputs", C.c_double),
        ("oz_listed", C.c_uint64), ("oz_reruns", C.c_uint64)]

    def as_dict(self) -> dict:
        return {n: getattr(self, n) for n, _ in self._fields_}


_lib = None


def load(path: str | os.PathLike | None = None) -> C.CDLL:
    """Load the library (once). Raises if it is missing or incomplete."""
    global _lib
    if _lib is not None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise ImportError(f"krystal_b200: CUDA library {p} is not built (run krystal_b200.build)")
    lib = C.CDLL(str(p))
    missing = [s for s in EXPORTS if not hasattr(lib, s)]
    if missing:
        raise ImportError(f"krystal_b200: {p} lacks exports {missing}")
    i = C.c_int
    lib.kc_abi_version.restype = C.c_uint32
    lib.kc_create.argtypes = [C.POINTER(KcConfig), C.POINTER(KcWeightsView), i, C.POINTER(P)]
    lib.kc_sync.argtypes = [P, C.POINTER(KcWeightsView), C.POINTER(KcChanges)]
    lib.kc_encode.argtypes = [P, C.POINTER(KcFrameView), P, P, P, C.c_uint32, C.c_uint32, u32p, u32p]
    lib.kc_select.argtypes = [P, C.POINTER(KcEncodedView), P, C.POINTER(KcMaskRule), P, P, P, P]
    lib.kc_forward_batch.argtypes = [P, C.POINTER(KcBatchView), C.POINTER(KcBatchOut)]
    lib.kc_select_batch.argtypes = [P, C.POINTER(KcBatchSelectView), C.POINTER(KcBatchOut)]
    lib.kc_forward_batch_device.argtypes = [P, C.POINTER(KcBatchView), C.POINTER(KcDeviceResult)]
    lib.kc_select_noalloc.argtypes = [P, C.c_uint32, C.c_uint32, P, P, P, P, P, P, P]
    lib.kc_set_precision.argtypes = [P, C.c_int, C.c_float]
    lib.kc_inject_wait_expiry.argtypes = [P, C.c_int]
    lib.kc_backward.argtypes = [P, C.POINTER(KcFrameView), P, P, i, C.c_double, C.POINTER(KcBackwardOut)]
    lib.kc_backward_batch_device.argtypes = [P, C.POINTER(KcBatchView), P, P, P, C.POINTER(KcBackwardResult)]
    lib.kc_learn_frame_stats.argtypes = [P, P, P]
    lib.kc_learn_accumulate.argtypes = [P, P, P, P]
    lib.kc_learn_plan.argtypes = [P, P, C.c_uint32, C.POINTER(KcLearnOptions), P, P, P, P]
    lib.kc_learn_accumulate_rows.argtypes = [P, P, P, P, P, P, P]
    lib.kc_learn_apply.argtypes = [P, P, P, P, P, C.POINTER(KcLearnOptions), P]
    lib.kc_copy_weights.argtypes = [P, C.c_uint64, C.c_uint64, P]
    lib.kc_stream_create.argtypes = [P, C.c_uint32, C.c_uint64, C.c_uint64, C.c_uint32, C.POINTER(P)]
    lib.kc_stream_push.argtypes = [P, C.POINTER(KcFrameView), P, P, C.POINTER(C.c_uint64)]
    lib.kc_stream_create_ex.argtypes = [P, C.c_uint32, C.c_uint64, C.c_uint64, C.c_uint32,
                                        C.POINTER(KcStreamOptions), C.POINTER(P)]
    lib.kc_stream_read_stats.argtypes = [P, i, C.POINTER(KcStreamStats)]
    lib.kc_stream_push_many.argtypes = [P, C.POINTER(KcBatchView), C.POINTER(C.c_uint64), C.POINTER(C.c_uint32)]
    lib.kc_stream_flush.argtypes = [P]
    lib.kc_load_checkpoint.argtypes = [P, P, C.c_uint64, C.POINTER(C.c_int)]
    lib.kc_save_checkpoint.argtypes = [P, P, C.c_uint64, C.POINTER(C.c_uint64)]
    lib.kc_stream_pending.argtypes = [P]
    lib.kc_stream_pending.restype = C.c_uint32
    lib.kc_stream_poll.argtypes = [P, i, C.POINTER(KcStreamResult)]
    lib.kc_stream_clock_ms.argtypes = []
    lib.kc_stream_clock_ms.restype = C.c_double
    lib.kc_stream_last_error.argtypes = [P]
    lib.kc_stream_last_error.restype = C.c_char_p
    lib.kc_stream_destroy.argtypes = [P]
    lib.kc_stream_destroy.restype = None
    lib.kc_set_stream.argtypes = [P, P]
    lib.kc_get_stream.argtypes = [P]
    lib.kc_get_stream.restype = P
    lib.kc_synchronize.argtypes = [P]
    lib.kc_profile.argtypes = [P, i]
    lib.kc_profile_read.argtypes = [P, C.POINTER(KcStageTimes), i]
    lib.kc_launch_count.argtypes = [P]
    lib.kc_launch_count.restype = C.c_uint64
    lib.kc_destroy.argtypes = [P]
    lib.kc_destroy.restype = None
    lib.kc_last_error.argtypes = [P]
    lib.kc_last_error.restype = C.c_char_p
    for name in ("kc_create", "kc_sync", "kc_encode", "kc_select", "kc_forward_batch", "kc_forward_batch_device",
                 "kc_set_stream", "kc_synchronize", "kc_profile", "kc_profile_read", "kc_select_noalloc",
                 "kc_set_precision", "kc_backward", "kc_backward_batch_device", "kc_learn_frame_stats",
                 "kc_learn_accumulate", "kc_stream_create", "kc_stream_push", "kc_stream_flush", "kc_stream_poll",
                 "kc_stream_push_many", "kc_load_checkpoint", "kc_save_checkpoint", "kc_select_batch",
                 "kc_inject_wait_expiry", "kc_learn_plan", "kc_learn_accumulate_rows", "kc_learn_apply",
                 "kc_copy_weights", "kc_stream_create_ex", "kc_stream_read_stats"):
        getattr(lib, name).restype = C.c_int
    _lib = lib
    return lib


def check(status: int, handle=None) -> None:
    if status != KC_OK:
        msg = load().kc_last_error(handle)
        raise KrystalCudaError(status, msg.decode() if msg else "")


def ptr(a) -> int | None:
    """Data pointer of a numpy array (or None)."""
    if a is None:
        return None
    return a.ctypes.data
