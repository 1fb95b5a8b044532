"""The oracle reproduces the committed golden fixtures bit for bit."""
import numpy as np
import pytest

from tests import golden_io as G


def test_test_records_golden(oracle):
    g, cfg, w, frame = G.test_records()
    assert G.sha(w.page) == str(g["weights_sha"])
    out = oracle.forward(cfg, w.page, frame)
    for k in ("field_states", "bank_keys", "bank_values", "query_output"):
        assert np.array_equal(out[k], g[k]), k
    sel = oracle.selector(out["query_output"], out["bank_keys"], out["bank_values"], g["grammar"], w.selector.wq,
                          w.selector.wk, 128)
    assert np.array_equal(sel["p"], g["p"]) and np.array_equal(sel["index"], g["index"])
    assert np.array_equal(sel["gather"], g["gather"])
    assert g["index"][0] < 2  # what the grammar forbids is never chosen


@pytest.mark.parametrize("name", G.BATCHES)
def test_batch_goldens(oracle, name):
    g, cfg, w, b, rule, u = G.batch(name)
    assert G.sha(w.page) == str(g["weights_sha"])
    res = oracle.forward_batch(cfg, w.page, b, rule=rule, uniforms=u, want_query_output=True)
    assert np.array_equal(res["p_off"], g["p_off"]) and np.array_equal(res["q_off"], g["q_off"])
    assert np.array_equal(res["index"], g["index"])
    assert np.array_equal(res["p"], g["p"])
    assert np.array_equal(res["query_output"], g["query_output"])


def test_batch_offsets_agree_with_host_packing(oracle):
    g, cfg, w, b, rule, u = G.batch("ragged_16_open")
    offs = b.offsets()
    o = oracle.batch_offsets(b)
    for k in ("p_off", "q_off", "r_off", "t_off"):
        assert np.array_equal(offs[k], o[k]), k
