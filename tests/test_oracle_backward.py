"""Pins the oracle's backward (forward/backward.ts:751-982 as host/gradients.ts
runs it) against central finite differences of the loss it differentiates:

    L = sum_q pointer(q) + mean_q 0.5 (pred_q - valence)^2
    pointer(q) = -log p[q, target]           (a target)
               = -log(1 - p[q, row])         (an AWAY target)

with p the selector's distribution under the selection mask and pred the
value head over [query output | gather | mean offered bank value].
"""
import numpy as np
import pytest

from krystal_b200.frame import pack_host_frame
from krystal_b200.model import BRAIN_FORWARD_CONFIG, create_brain_forward_weights, weight_layout
from krystal_b200.session import selection_mask

H = 128


def setup(seed=7):
    cfg = BRAIN_FORWARD_CONFIG.with_token_rows(np.arange(4096, dtype=np.uint32) % 64)
    w = create_brain_forward_weights(cfg, seed)
    rng = np.random.default_rng(seed)
    recs = [dict(schemaId=int(rng.integers(0, 8)), band=int(rng.choice([0, 1, 2, 3])),
                 tokens=[int(t) for t in rng.integers(1, 60, rng.integers(1, 9))]) for _ in range(9)]
    recs += [dict(query=True, tokens=[int(t) for t in rng.integers(1, 60, 3)]) for _ in range(3)]
    frame = pack_host_frame(recs)
    mask = selection_mask(frame.active, lambda q, slot: (q + slot) % 4 != 0)
    return cfg, w, frame, mask


def loss_of(oracle, cfg, page, frame, mask, targets, valence):
    fw = oracle.forward(cfg, page, frame.gpu)
    lay = weight_layout(cfg)
    qo = fw["query_output"].astype(np.float64).reshape(-1, H)
    bk = fw["bank_keys"].astype(np.float64).reshape(-1, H)
    bv = fw["bank_values"].astype(np.float64).reshape(-1, H)
    wq = page[lay.selector_wq:lay.selector_wq + H * H].astype(np.float64).reshape(H, H)
    wk = page[lay.selector_wk:lay.selector_wk + H * H].astype(np.float64).reshape(H, H)
    wv = page[lay.value_head:lay.total].astype(np.float64)
    q, r = qo.shape[0], bk.shape[0]
    m = mask.reshape(q, r).astype(np.float64)
    s = (qo @ wq.T) @ (bk @ wk.T).T / np.sqrt(H) + m
    p = np.exp(s - s.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    gather = p @ bv
    offered = np.stack([bv[m[i] > -1e29].mean(0) for i in range(q)])
    pred = np.concatenate([qo, gather, offered], 1) @ wv
    L = 0.5 * np.mean((pred - valence) ** 2)
    for i, tg in enumerate(targets):
        if tg == 0xFFFFFFFF:
            continue
        if tg & 0x80000000:
            L -= np.log(1 - p[i, tg & 0x7FFFFFFF])
        else:
            L -= np.log(p[i, tg])
    return L


def fd(oracle, cfg, w, frame, mask, targets, valence, idx, eps):
    page = w.page.copy()
    page[idx] += eps
    lp = loss_of(oracle, cfg, page, frame, mask, targets, valence)
    page[idx] -= 2 * eps
    lm = loss_of(oracle, cfg, page, frame, mask, targets, valence)
    return (lp - lm) / (2 * eps)


@pytest.mark.parametrize("targets", [[1, 0xFFFFFFFF, 4], [0x80000002, 4, 0xFFFFFFFF]])
def test_backward_gradients_match_finite_differences(oracle, targets):
    cfg, w, frame, mask = setup()
    valence = 0.3
    bw = oracle.backward(cfg, w.page, frame.gpu, mask, np.array(targets, np.uint32), valence)
    lay = weight_layout(cfg)
    rng = np.random.default_rng(1)
    # selector Wq / Wk: the largest few entries and a few random ones
    for name, base in (("d_selector_wq", lay.selector_wq), ("d_selector_wk", lay.selector_wk)):
        g = bw[name]
        for k in list(np.argsort(-np.abs(g))[:3]) + list(rng.integers(0, H * H, 2)):
            num = fd(oracle, cfg, w, frame, mask, targets, valence, base + int(k), 1e-3)
            assert abs(num - g[k]) <= 0.02 * abs(g).max() + 1e-6, (name, k, num, g[k])
    # pool query rows
    g = bw["d_pool"]
    for k in list(np.argsort(-np.abs(g))[:3]):
        num = fd(oracle, cfg, w, frame, mask, targets, valence, lay.pool + int(k), 1e-3)
        assert abs(num - g[k]) <= 0.03 * abs(g).max() + 1e-6, ("d_pool", k, num, g[k])
    # value head
    g = bw["d_value_wv"]
    for k in list(np.argsort(-np.abs(g))[:3]):
        num = fd(oracle, cfg, w, frame, mask, targets, valence, lay.value_head + int(k), 1e-3)
        assert abs(num - g[k]) <= 0.02 * abs(g).max() + 1e-6, ("d_value_wv", k, num, g[k])
    # field states: a token table row used by exactly one token carries that token's gradient
    act = frame.active
    ids = frame.gpu.token_ids[act.active_tokens]
    rows = cfg.token_rows[ids]
    uniq, counts = np.unique(rows, return_counts=True)
    dfs = bw["d_field_states"].reshape(-1, H)
    for row in uniq[counts == 1][:2]:
        t = int(np.nonzero(rows == row)[0][0])
        for dd in list(np.argsort(-np.abs(dfs[t]))[:2]):
            num = fd(oracle, cfg, w, frame, mask, targets, valence, int(row) * H + int(dd), 1e-3)
            assert abs(num - dfs[t, dd]) <= 0.03 * np.abs(dfs).max() + 1e-6, ("d_field_states", t, dd, num)


def test_backward_without_targets_or_valence_is_zero(oracle):
    cfg, w, frame, mask = setup(3)
    bw = oracle.backward(cfg, w.page, frame.gpu, mask, None, None)
    for k in ("d_selector_wq", "d_selector_wk", "d_pool", "d_field_states", "d_value_wv"):
        assert not bw[k].any(), k
    assert bw["value_loss"] == 0
    fw = oracle.forward(cfg, w.page, frame.gpu)
    sel = oracle.selector(fw["query_output"], fw["bank_keys"], fw["bank_values"], mask, w.selector.wq,
                          w.selector.wk, 128)
    assert np.array_equal(bw["policy"], sel["p"])


def test_value_loss_and_prediction(oracle):
    cfg, w, frame, mask = setup(5)
    bw = oracle.backward(cfg, w.page, frame.gpu, mask, None, 1.5)
    pred = bw["value_prediction"].astype(np.float64)
    assert abs(bw["value_loss"] - np.mean(0.5 * (pred - 1.5) ** 2)) < 1e-9
