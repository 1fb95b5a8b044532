"""kc_select_noalloc against kc_select, through the C ABI, on two calls in a row.

kc_select_noalloc is for callers that cannot allocate device memory where
they select (inside CUDA stream capture, in allocation-free real-time loops,
or under an external memory pool); it keeps its scratch in a static device
array. The test owns its device buffers (torch allocates them here, in the
test, not in the entry point) and compares both calls with the allocating
entry point and with the oracle's selector: selected indices exact, p within
the parity tolerance. A batch left resident for kc_select_batch must survive
a no-alloc call, which never touches the handle's workspace.
This file is collected last so a stop-at-first-failure run has already run
every other test; it also passes alone in a fresh process.
"""
import numpy as np
import pytest

from krystal_b200 import abi, synth
from krystal_b200.backend import CudaBrainBackend, MaskRule
from krystal_b200.frame import pack_host_frame
from krystal_b200.model import BRAIN_FORWARD_CONFIG, create_brain_forward_weights

pytestmark = pytest.mark.gpu

P_TOL = 1e-4


def test_noalloc_select_matches_select_twice_in_a_row(oracle):
    torch = pytest.importorskip("torch")
    cfg = BRAIN_FORWARD_CONFIG.with_token_rows(np.arange(4096, dtype=np.uint32) % 64)
    w = create_brain_forward_weights(cfg, 5)
    be = CudaBrainBackend(cfg, w, 0)
    rng = np.random.default_rng(17)
    try:
        for call in range(2):
            nb, nq = (37, 5) if call == 0 else (120, 9)
            recs = [dict(schemaId=int(rng.integers(0, 9)), tokens=[int(t) for t in rng.integers(1, 4000, rng.integers(1, 9))])
                    for _ in range(nb)] + [dict(query=True, tokens=[int(rng.integers(1, 4000))]) for _ in range(nq)]
            enc = be.encode(pack_host_frame(recs))
            mask = None
            if call == 0:
                mask = np.where(rng.random(nq * nb) < 0.3, np.float32(-1e30), np.float32(0)).astype(np.float32)
                mask[:nb] = -1e30  # one question with everything blocked
            want = be.select(enc, mask=mask)
            ref = oracle.selector(enc.query_output, enc.bank_keys, enc.bank_values, mask, w.selector.wq,
                                  w.selector.wk, 128)
            assert np.array_equal(want.index, ref["index"]), call
            dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
            d_q, d_k, d_v = dev(enc.query_output), dev(enc.bank_keys), dev(enc.bank_values)
            d_m = dev(mask) if mask is not None else None
            d_p = torch.full((nq * nb,), float("nan"), dtype=torch.float32, device="cuda")
            d_i = torch.zeros(nq, dtype=torch.int32, device="cuda")
            d_g = torch.zeros(nq * 128, dtype=torch.float32, device="cuda")
            torch.cuda.synchronize()
            be.select_noalloc(nq, nb, d_q.data_ptr(), d_k.data_ptr(), d_v.data_ptr(),
                              d_m.data_ptr() if d_m is not None else None, d_p.data_ptr(), d_i.data_ptr(),
                              d_g.data_ptr())
            be.synchronize()
            p = d_p.cpu().numpy()
            idx = d_i.cpu().numpy().view(np.uint32)
            assert np.array_equal(idx, want.index), call
            assert np.array_equal(idx, ref["index"]), call
            assert np.abs(p - ref["p"]).max() <= P_TOL, call
            assert np.abs(p - want.p).max() <= P_TOL, call
            assert np.abs(d_g.cpu().numpy() - want.gather).max() <= 1e-5, call
            if call == 0:
                assert idx[0] == abi.KC_NO_SELECTION and not p[:nb].any()
        with pytest.raises(abi.KrystalCudaError) as e:
            be.select_noalloc(257, 4, d_q.data_ptr(), d_k.data_ptr(), None, None, d_p.data_ptr(), d_i.data_ptr())
        assert e.value.status == abi.KC_ERR_CAPACITY
    finally:
        be.destroy()


def test_resident_batch_survives_a_noalloc_call():
    """kc_select_batch reselects the last forward_batch's batch; a no-alloc
    selection in between must leave that batch usable."""
    torch = pytest.importorskip("torch")
    wl = synth.WORKLOADS["ragged_4096"]
    cfg = synth.workload_config(wl)
    w = synth.workload_weights(cfg, wl.vocab)
    be = CudaBrainBackend(cfg, w, 0)
    try:
        batch = synth.make_batch(wl, seed=61, frames=12)
        rule = MaskRule(*synth.make_rule(batch, seed=62))
        first = be.forward_batch(batch)
        before = be.select_batch(rule=rule)
        d_q = torch.randn(3 * 128, dtype=torch.float32, device="cuda")
        d_k = torch.randn(20 * 128, dtype=torch.float32, device="cuda")
        d_p = torch.empty(60, dtype=torch.float32, device="cuda")
        d_i = torch.empty(3, dtype=torch.int32, device="cuda")
        torch.cuda.synchronize()
        be.select_noalloc(3, 20, d_q.data_ptr(), d_k.data_ptr(), None, None, d_p.data_ptr(), d_i.data_ptr())
        be.synchronize()
        after = be.select_batch(rule=rule)
        again = be.select_batch()
    finally:
        be.destroy()
    assert np.array_equal(before["index"], after["index"]) and np.array_equal(before["p"], after["p"])
    assert np.array_equal(again["index"], first["index"]) and np.array_equal(again["p"], first["p"])
