"""GPU tests of the exact path's products on the int8 tensor cores
(csrc/ozaki.cuh). matmulOracle (forward/oracle.ts:114-125) stores f32 of one
f64 chain per output; the int8 product settles every output whose error
interval rounds to one f32 and hands the rest to the sequential chain, so the
exact batch must equal, bit for bit, the same batch with every product on the
FP64 kernel (KC_NO_OZAKI=1), and the oracle. A list too short for the outputs
to settle (KC_OZAKI_LIST_CAP) sends the forward back through the FP64 kernel
with the same results; an expired wait fails the call and leaves the handle
usable.
"""
import os

import numpy as np
import pytest

from krystal_b200 import abi, synth
from krystal_b200.backend import CudaBrainBackend

pytestmark = pytest.mark.gpu


def make_backend(cfg, w, env: dict):
    saved = {k: os.environ.pop(k, None) for k in ("KC_NO_OZAKI", "KC_OZAKI_LIST_CAP")}
    try:
        os.environ.update(env)
        return CudaBrainBackend(cfg, w, 0)
    finally:
        for k in ("KC_NO_OZAKI", "KC_OZAKI_LIST_CAP"):
            os.environ.pop(k, None)
            if saved[k] is not None:
                os.environ[k] = saved[k]


@pytest.fixture(scope="module")
def ragged():
    wl = synth.WORKLOADS["ragged_4096"]
    cfg = synth.workload_config(wl)
    w = synth.workload_weights(cfg, wl.vocab)
    return wl, cfg, w


def exact_batch(be, batch):
    be.set_precision("exact")
    be.profile(True)
    be.profile_read(reset=True)
    res = be.forward_batch(batch)
    prof = be.profile_read(reset=True)
    be.profile(False)
    return res, prof


def assert_same(a, b):
    assert np.array_equal(a["index"], b["index"])
    assert np.array_equal(a["p"].view(np.uint32), b["p"].view(np.uint32))
    assert np.array_equal(a["p_off"], b["p_off"]) and np.array_equal(a["q_off"], b["q_off"])


@pytest.mark.parametrize("token_scale", [1.0, 64.0])
def test_int8_products_equal_the_fp64_kernel(ragged, oracle, token_scale):
    wl, cfg, w = ragged
    if token_scale != 1.0:  # activations 64x larger: the slices' exponents move, the results must not
        w = synth.workload_weights(cfg, wl.vocab)
        w.embeddings[:wl.vocab * cfg.hidden_size] *= np.float32(token_scale)
    batch = synth.make_batch(wl, seed=41, frames=192)
    oz = make_backend(cfg, w, {})
    fp = make_backend(cfg, w, {"KC_NO_OZAKI": "1"})
    try:
        got, prof = exact_batch(oz, batch)
        want, prof_fp = exact_batch(fp, batch)
    finally:
        oz.destroy()
        fp.destroy()
    assert_same(got, want)
    assert prof["oz_products"] > 0 and prof["oz_reruns"] == 0
    assert prof_fp["oz_products"] == 0
    listed = prof["oz_listed"] / prof["oz_outputs"]
    print(f"token rows x{token_scale}: {prof['oz_products']} products, {prof['oz_outputs']:.0f} outputs, "
          f"{prof['oz_listed']} listed ({listed:.2e})")
    assert listed < 0.01
    small = batch.subset(list(range(6)))
    ref = oracle.forward_batch(cfg, w.page, small)
    head = {"p": got["p"][: int(got["p_off"][6])], "index": got["index"][: int(got["q_off"][6])]}
    assert np.array_equal(head["index"], ref["index"])
    assert np.array_equal(head["p"].view(np.uint32), np.asarray(ref["p"], np.float32).view(np.uint32))


def test_a_full_list_reruns_on_the_fp64_kernel(ragged):
    wl, cfg, w = ragged
    batch = synth.make_batch(wl, seed=42, frames=64)
    oz = make_backend(cfg, w, {"KC_OZAKI_LIST_CAP": "0"})
    fp = make_backend(cfg, w, {"KC_NO_OZAKI": "1"})
    try:
        got, prof = exact_batch(oz, batch)
        want, _ = exact_batch(fp, batch)
    finally:
        oz.destroy()
        fp.destroy()
    assert prof["oz_reruns"] == 1  # every listed output overflows a list of length 0
    assert_same(got, want)


def test_expired_wait_in_the_int8_product(ragged):
    wl, cfg, w = ragged
    batch = synth.make_batch(wl, seed=43, frames=48)  # enough tokens for the encoder's products to take the int8 path
    be = make_backend(cfg, w, {})
    try:
        be.set_precision("exact")
        before = be.forward_batch(batch)
        be.inject_wait_expiry("exact_gemm")
        with pytest.raises(abi.KrystalCudaError) as e:
            be.forward_batch(batch)
        assert e.value.status == abi.KC_ERR_TIMEOUT and "wait expired" in e.value.message
        after = be.forward_batch(batch)
    finally:
        be.destroy()
    assert_same(after, before)
