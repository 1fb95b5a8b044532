"""An independent numpy restatement of the reference forward, for cross-checks.

Vectorised over rows with numpy's own summation order, f32 stores where the
reference stores into a Float32Array. It is NOT bit-identical to the oracle
(numpy sums in another order); it agrees to a few f32 ulps, which is what the
cross-check asserts. Reference: packages/krystal/src/forward/oracle.ts.
"""
import numpy as np

from krystal_b200.frame import record_ranges
from krystal_b200.model import embedding_table_bases


def softmax_rows(s):  # softmaxRow over the last axis, f32 in, f32 out
    s = s.astype(np.float64)
    e = np.exp(s - s.max(axis=-1, keepdims=True))
    ef = e.astype(np.float32).astype(np.float64)
    inv = 1.0 / np.maximum(e.sum(axis=-1, keepdims=True), 1e-20)
    return (ef * inv).astype(np.float32)


def mm(x, w, out_dim, in_dim):
    return (x.astype(np.float64).reshape(-1, in_dim) @ w.astype(np.float64).reshape(out_dim, in_dim).T).astype(
        np.float32)


def forward(config, weights, frame, word_ids=None, alpha=0.0):
    h, heads, hd, f = config.hidden_size, config.head_count, config.head_dim, config.ffn_size
    g, act = frame.gpu, frame.active
    b = embedding_table_bases(config)
    E = weights.embeddings.astype(np.float64)
    ft = act.active_tokens.astype(np.int64)
    slot, local = ft >> 3, ft & 7
    rows = config.token_rows
    tok = rows[g.token_ids[ft]].astype(np.int64)
    role = rows[g.field_roles[ft]].astype(np.int64)
    stream = act.stream_ids[slot].astype(np.int64)
    d = np.arange(h)
    x = (E[b.token + tok[:, None] * h + d] + E[b.field + role[:, None] * h + d]
         + E[b.schema + g.schema_ids[slot].astype(np.int64)[:, None] * h + d]
         + E[b.band + g.band_ids[slot].astype(np.int64)[:, None] * h + d]
         + E[b.stream + stream[:, None] * h + d] + E[b.pos + local[:, None] * h + d]).astype(np.float32)
    start, count = record_ranges(act)
    t = x.shape[0]
    # the same-word bias (WordBias): f32 alpha between two tokens of one record with one valid word id
    words = None if word_ids is None or alpha == 0 else np.asarray(word_ids, np.uint32)[ft]
    a32 = float(np.float32(alpha))
    for blk in weights.enc:
        q, k, v = mm(x, blk.wq, h, h), mm(x, blk.wk, h, h), mm(x, blk.wv, h, h)
        out = np.zeros((t, h), dtype=np.float32)
        for i in range(t):
            s0, c = int(start[i]), int(count[i])
            for hh in range(heads):
                sl = slice(hh * hd, (hh + 1) * hd)
                bias = 0.0
                if words is not None:
                    wj = words[s0:s0 + c]
                    bias = np.where((wj == words[i]) & (words[i] != 0xFFFFFFFF), a32, 0.0)
                sc = (k[s0:s0 + c, sl].astype(np.float64) @ q[i, sl].astype(np.float64) / np.sqrt(hd)
                      + bias).astype(np.float32)
                p = softmax_rows(sc)
                out[i, sl] = (p.astype(np.float64) @ v[s0:s0 + c, sl].astype(np.float64)).astype(np.float32)
        x = (x + out).astype(np.float32)
        hid = np.maximum(mm(x, blk.w1, f, h), 0)
        x = (x + mm(hid, blk.w2, h, f)).astype(np.float32)

    def pool(slots):
        keys = np.zeros((len(slots), h), dtype=np.float32)
        vals = np.zeros((len(slots), h), dtype=np.float32)
        P = weights.pool.astype(np.float64).reshape(2, h)
        for n, s in enumerate(slots):
            s0, c = int(act.record_compact_offset[s]), int(act.record_compact_count[s])
            if c == 0:
                continue
            xs = x[s0:s0 + c].astype(np.float64)
            sc = (xs @ P.T / np.sqrt(h)).astype(np.float32)
            pk, pv = softmax_rows(sc[:, 0]), softmax_rows(sc[:, 1])
            keys[n] = (pk.astype(np.float64) @ xs).astype(np.float32)
            vals[n] = (pv.astype(np.float64) @ xs).astype(np.float32)
        return keys, vals

    bk, bv = pool(act.bank_records.tolist())
    _, qv = pool(act.query_records.tolist())
    query = qv.copy()
    for blk in weights.mixer:
        mq, mk, mv = mm(query, blk.wq, h, h), mm(bk, blk.wk, h, h), mm(bv, blk.wv, h, h)
        out = np.zeros_like(query)
        for hh in range(heads):
            sl = slice(hh * hd, (hh + 1) * hd)
            sc = (mq[:, sl].astype(np.float64) @ mk[:, sl].astype(np.float64).T / np.sqrt(hd)).astype(np.float32)
            p = softmax_rows(sc)
            out[:, sl] = (p.astype(np.float64) @ mv[:, sl].astype(np.float64)).astype(np.float32)
        query = (query + out).astype(np.float32)
        hid = np.maximum(mm(query, blk.w1, f, h), 0)
        query = (query + mm(hid, blk.w2, h, f)).astype(np.float32)
    return {"field_states": x.reshape(-1), "bank_keys": bk.reshape(-1), "bank_values": bv.reshape(-1),
            "query_output": query.reshape(-1)}


def selector(query, bank_keys, mask, wq, wk, h):
    qp, kp = mm(query, wq, h, h), mm(bank_keys, wk, h, h)
    sc = (qp.astype(np.float64) @ kp.astype(np.float64).T / np.sqrt(h)
          + (0 if mask is None else mask.reshape(qp.shape[0], -1))).astype(np.float32)
    return softmax_rows(sc).reshape(-1)
