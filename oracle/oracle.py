"""ctypes binding to the C++ oracle (oracle/krystal_oracle.cpp).

TEST INFRASTRUCTURE ONLY: the checker. Imported by tests/, by the smoke
check and by the benchmark's CPU-baseline leg and reference arm — never by
the product package.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "libkrystal_oracle.so"


class KoDims(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in (
        "hidden", "heads", "head_dim", "ffn", "enc_blocks", "mixer_blocks", "token_space", "field_space",
        "schema_space", "band_space", "stream_space", "pos_space", "route_kinds")]


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        _lib = C.CDLL(str(LIB_PATH))
        P = C.c_void_p
        u32, u64, i32 = C.c_uint32, C.c_uint64, C.c_int32
        _lib.ko_weight_count.restype = u64
        _lib.ko_weight_count.argtypes = [P]
        _lib.ko_weight_offset.restype = u64
        _lib.ko_weight_offset.argtypes = [P, C.c_int]
        _lib.ko_create_weights.argtypes = [P, u32, P]
        _lib.ko_mulberry32.argtypes = [u32, u32, P]
        _lib.ko_matmul.argtypes = [P, P, u32, u32, u32, P]
        _lib.ko_softmax_row.argtypes = [P, u32]
        _lib.ko_sample_row.restype = i32
        _lib.ko_sample_row.argtypes = [P, u32, C.c_double]
        _lib.ko_compile_active.restype = u32
        _lib.ko_compile_active.argtypes = [u32, P, P, P, P, P, P, P, P, P, P, P, P]
        _lib.ko_forward.restype = C.c_int
        _lib.ko_forward.argtypes = [P, P, P, u32, u32, P, P, P, P, P, P, P, P, P, P, P, P, P, C.c_float]
        _lib.ko_selector.argtypes = [P, P, P, P, P, P, u32, u32, u32, P, P, P, P]
        _lib.ko_selection_mask_rule.argtypes = [u32, u32, P, P, P, P, P, P]
        _lib.ko_forward_batch.restype = C.c_int
        _lib.ko_forward_batch.argtypes = [P, P, P, u32, u32, P, P, P, P, P, P, P, P, C.c_int, P, P, P, P, P, P,
                                          C.c_float]
        _lib.ko_batch_offsets.argtypes = [u32, P, P, P, P, P, P, P]
        _lib.ko_max_threads.restype = C.c_int
        _lib.ko_backward.restype = C.c_int
        _lib.ko_backward.argtypes = [P, P, P, u32, u32, P, P, P, P, P, P, P, C.c_int, C.c_double, P, P, P, P, P, P,
                                     P, P]
    return _lib


def _u32(a):
    return None if a is None else np.ascontiguousarray(a, dtype=np.uint32)


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def dims_of(config) -> KoDims:
    return KoDims(config.hidden_size, config.head_count, config.head_dim, config.ffn_size, config.encoder_blocks,
                  config.mixer_blocks, config.token_space, config.field_space, config.schema_space,
                  config.band_space, config.stream_space, config.pos_space, config.route_kind_count)


def weight_count(config) -> int:
    d = dims_of(config)
    return int(lib().ko_weight_count(C.byref(d)))


WEIGHT_PARTS = ("embeddings", "encoder", "pool", "mixer", "selector_wq", "selector_wk", "decision_head", "value_head")


def weight_offset(config, part: str) -> int:
    """Element offset of a part of the weight page (model.ts:233-265 order)."""
    d = dims_of(config)
    return int(lib().ko_weight_offset(C.byref(d), WEIGHT_PARTS.index(part)))


def create_weights(config, seed: int) -> np.ndarray:
    d = dims_of(config)
    out = np.empty(weight_count(config), dtype=np.float32)
    lib().ko_create_weights(C.byref(d), seed, _p(out))
    return out


def mulberry32(seed: int, n: int) -> np.ndarray:
    out = np.empty(n, dtype=np.float64)
    lib().ko_mulberry32(seed, n, _p(out))
    return out


def matmul(x, w, out_dim: int, in_dim: int) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows = x.size // in_dim
    y = np.empty(rows * out_dim, dtype=np.float32)
    lib().ko_matmul(_p(x), _p(w), rows, out_dim, in_dim, _p(y))
    return y


def softmax_row(v) -> np.ndarray:
    v = np.array(v, dtype=np.float32)
    lib().ko_softmax_row(_p(v), v.size)
    return v


def sample_row(p, uniform: float) -> int:
    p = np.ascontiguousarray(p, dtype=np.float32)
    return int(lib().ko_sample_row(_p(p), p.size, uniform))


def compile_active(token_ids, band_ids, active_record_indices=None) -> dict:
    token_ids = np.ascontiguousarray(token_ids, dtype=np.uint32)
    band_ids = np.ascontiguousarray(band_ids, dtype=np.uint32)
    slots = band_ids.size
    ari = None if active_record_indices is None else np.ascontiguousarray(active_record_indices, dtype=np.uint32)
    at = np.empty(slots * 8, dtype=np.uint32)
    off = np.empty(slots, dtype=np.uint32)
    cnt = np.empty(slots, dtype=np.uint32)
    st = np.empty(slots, dtype=np.uint32)
    bank = np.empty(slots, dtype=np.uint32)
    qry = np.empty(slots, dtype=np.uint32)
    r, q, n = C.c_uint32(), C.c_uint32(), C.c_uint32()
    t = lib().ko_compile_active(slots, _p(token_ids), _p(band_ids), _p(ari), _p(at), _p(off), _p(cnt), _p(st),
                                _p(bank), _p(qry), C.byref(r), C.byref(q), C.byref(n))
    return {"active_tokens": at[:t].copy(), "record_compact_offset": off, "record_compact_count": cnt,
            "stream_ids": st, "bank_records": bank[:r.value].copy(), "query_records": qry[:q.value].copy(),
            "active_count": n.value}


def forward(config, weights_page: np.ndarray, frame, mixer_mask=None, word_ids=None, alpha: float = 0.0) -> dict:
    """brainForwardOracle on one BrainFrameGpu-like object (fields token_ids, ...).
    word_ids [slots*8] / alpha: the same-word bias on the encoder's record mask."""
    d = dims_of(config)
    h = config.hidden_size
    act = compile_active(frame.token_ids, frame.band_ids, frame.active_record_indices)
    t, r, q = act["active_tokens"].size, act["bank_records"].size, act["query_records"].size
    out = {k: np.zeros(n * h, dtype=np.float32) for k, n in (
        ("field_states", t), ("bank_keys", r), ("bank_values", r), ("query_keys", q), ("query_values", q),
        ("query_output", q))}
    rows = np.ascontiguousarray(config.token_rows, dtype=np.uint32)
    mm = None if mixer_mask is None else np.ascontiguousarray(mixer_mask, dtype=np.float32)
    rc = lib().ko_forward(C.byref(d), _p(weights_page), _p(rows), rows.size, frame.schema_ids.size,
                          _p(frame.token_ids), _p(frame.field_roles), _p(frame.schema_ids), _p(frame.band_ids),
                          _p(frame.active_record_indices), _p(mm), _p(out["field_states"]), _p(out["bank_keys"]),
                          _p(out["bank_values"]), _p(out["query_keys"]), _p(out["query_values"]),
                          _p(out["query_output"]), _p(_u32(word_ids)), float(alpha))
    if rc != 0:
        raise ValueError("oracle: frame references a row outside its table")
    out.update(t=t, r=r, q=q, active=act)
    return out


def selector(query, bank_keys, bank_values, mask, wq, wk, h: int, uniforms=None) -> dict:
    q = query.size // h
    r = bank_keys.size // h
    p = np.empty(q * r, dtype=np.float32)
    gather = np.empty(q * h, dtype=np.float32)
    index = np.empty(q, dtype=np.uint32)
    m = None if mask is None else np.ascontiguousarray(mask, dtype=np.float32)
    u = None if uniforms is None else np.ascontiguousarray(uniforms, dtype=np.float64)
    lib().ko_selector(_p(np.ascontiguousarray(query, np.float32)), _p(np.ascontiguousarray(bank_keys, np.float32)),
                      _p(np.ascontiguousarray(bank_values, np.float32)), _p(m),
                      _p(np.ascontiguousarray(wq, np.float32)), _p(np.ascontiguousarray(wk, np.float32)), q, r, h,
                      _p(u), _p(p), _p(gather), _p(index))
    return {"p": p, "gather": gather, "index": index}


def selection_mask_rule(bank_records, schema_ids, band_ids, schema_allow, band_allow, q: int) -> np.ndarray:
    r = bank_records.size
    mask = np.empty(q * r, dtype=np.float32)
    lib().ko_selection_mask_rule(q, r, _p(np.ascontiguousarray(bank_records, np.uint32)),
                                 _p(np.ascontiguousarray(schema_ids, np.uint32)),
                                 _p(np.ascontiguousarray(band_ids, np.uint32)),
                                 _p(np.ascontiguousarray(schema_allow, np.uint32)),
                                 _p(np.ascontiguousarray(band_allow, np.uint32)), _p(mask))
    return mask


def batch_offsets(batch) -> dict:
    F = batch.frames
    p_off = np.empty(F + 1, dtype=np.uint64)
    q_off = np.empty(F + 1, dtype=np.uint64)
    r_off = np.empty(F + 1, dtype=np.uint64)
    t_off = np.empty(F + 1, dtype=np.uint64)
    lib().ko_batch_offsets(F, _p(batch.rec_off), _p(batch.token_ids), _p(batch.band_ids), _p(p_off), _p(q_off),
                           _p(r_off), _p(t_off))
    return {"p_off": p_off, "q_off": q_off, "r_off": r_off, "t_off": t_off}


def forward_batch(config, weights_page: np.ndarray, batch, rule=None, uniforms=None, threads: int = 0,
                  want_query_output: bool = False, word_ids=None, alpha: float = 0.0) -> dict:
    d = dims_of(config)
    offs = batch_offsets(batch)
    F = batch.frames
    p = np.empty(int(offs["p_off"][-1]), dtype=np.float32)
    index = np.empty(int(offs["q_off"][-1]), dtype=np.uint32)
    qout = np.empty(int(offs["q_off"][-1]) * config.hidden_size, dtype=np.float32) if want_query_output else None
    rows = np.ascontiguousarray(config.token_rows, dtype=np.uint32)
    sa, ba = (None, None) if rule is None else rule
    u = None if uniforms is None else np.ascontiguousarray(uniforms, dtype=np.float64)
    wid = _u32(word_ids)
    rc = lib().ko_forward_batch(C.byref(d), _p(weights_page), _p(rows), rows.size, F, _p(batch.rec_off),
                                _p(batch.token_ids), _p(batch.field_roles), _p(batch.schema_ids),
                                _p(batch.band_ids), _p(sa), _p(ba), _p(u), threads, _p(offs["p_off"]),
                                _p(offs["q_off"]), _p(p), _p(index), _p(qout), _p(wid), float(alpha))
    if rc != 0:
        raise ValueError("oracle: a frame references a row outside its table")
    out = {"p": p, "index": index, **offs}
    if qout is not None:
        out["query_output"] = qout
    return out


def backward(config, weights_page: np.ndarray, frame, selection, targets=None, valence=None) -> dict:
    """brainBackwardOracle as a session runs it (BackwardResult fields)."""
    d = dims_of(config)
    h = config.hidden_size
    act = compile_active(frame.token_ids, frame.band_ids, frame.active_record_indices)
    t, r, q = act["active_tokens"].size, act["bank_records"].size, act["query_records"].size
    out = {"policy": np.zeros(max(1, q * r), np.float32), "value_prediction": np.zeros(max(1, q), np.float32),
           "d_selector_wq": np.zeros(h * h, np.float32), "d_selector_wk": np.zeros(h * h, np.float32),
           "d_pool": np.zeros(2 * h, np.float32), "d_field_states": np.zeros(max(1, t * h), np.float32),
           "d_value_wv": np.zeros(3 * h, np.float32)}
    loss = C.c_double()
    rows = np.ascontiguousarray(config.token_rows, dtype=np.uint32)
    sel = np.ascontiguousarray(selection, dtype=np.float32)
    tg = None if targets is None else np.ascontiguousarray(targets, dtype=np.uint32)
    rc = lib().ko_backward(C.byref(d), _p(weights_page), _p(rows), rows.size, frame.schema_ids.size,
                           _p(frame.token_ids), _p(frame.field_roles), _p(frame.schema_ids), _p(frame.band_ids),
                           _p(frame.active_record_indices), _p(sel), _p(tg), int(valence is not None),
                           float(valence or 0.0), _p(out["policy"]), _p(out["value_prediction"]), C.byref(loss),
                           _p(out["d_selector_wq"]), _p(out["d_selector_wk"]), _p(out["d_pool"]),
                           _p(out["d_field_states"]), _p(out["d_value_wv"]))
    if rc != 0:
        raise ValueError("oracle: frame references a row outside its table")
    out["policy"] = out["policy"][:q * r]
    out["value_prediction"] = out["value_prediction"][:q]
    out["d_field_states"] = out["d_field_states"][:t * h]
    out.update(value_loss=loss.value, t=t, r=r, q=q, active=act)
    return out


def max_threads() -> int:
    return int(lib().ko_max_threads())


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return os.uname().machine
