"""The bounded-wait failure path of the tensor-core kernels, run on purpose.

Every wait in the tcgen05 pipelines (the fused encoder attention, the fused
feed-forward, the projection GEMM) is bounded. When one expires the kernel
raises an error word, every warp role leaves (copies and MMAs already issued
are drained first), TMEM is freed, and the batch call returns KC_ERR_TIMEOUT.
kc_inject_wait_expiry makes the next launch of one kernel behave as if its
producer's first wait had expired, before it issues any copy, so nothing
actually hangs or faults. The same handle must then run the batch normally
and give the results it gave before.
"""
import numpy as np
import pytest

from krystal_b200 import abi, synth
from krystal_b200.backend import CudaBrainBackend

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kernel", ["attn", "ffn", "gemm"])
def test_expired_wait_returns_timeout_and_the_handle_recovers(oracle, kernel):
    wl = synth.WORKLOADS["ragged_4096"]
    cfg = synth.workload_config(wl)
    w = synth.workload_weights(cfg, wl.vocab)
    batch = synth.make_batch(wl, seed=31, frames=24)
    be = CudaBrainBackend(cfg, w, 0)
    try:
        before = be.forward_batch(batch)
        be.inject_wait_expiry(kernel)
        with pytest.raises(abi.KrystalCudaError) as e:
            be.forward_batch(batch)
        assert e.value.status == abi.KC_ERR_TIMEOUT
        assert "wait expired" in e.value.message
        after = be.forward_batch(batch)
        again = be.forward_batch(batch)
    finally:
        be.destroy()
    want = oracle.forward_batch(cfg, w.page, batch)
    for res in (before, after, again):
        assert np.array_equal(res["index"], want["index"])
        assert np.abs(res["p"] - want["p"]).max() <= 1e-4
    assert np.array_equal(after["p"], before["p"]) and np.array_equal(again["p"], before["p"])


def test_injection_is_refused_for_an_unknown_kernel():
    wl = synth.WORKLOADS["ragged_4096"]
    cfg = synth.workload_config(wl)
    be = CudaBrainBackend(cfg, synth.workload_weights(cfg, wl.vocab), 0)
    try:
        with pytest.raises(abi.KrystalCudaError) as e:
            abi.check(be._lib.kc_inject_wait_expiry(be._h, 7), be._h)
        assert e.value.status == abi.KC_ERR_INVALID_ARG
    finally:
        be.destroy()
