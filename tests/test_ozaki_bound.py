"""The error bound behind the exact path's int8 products (csrc/ozaki.cuh),
checked on the CPU with a numpy model of the same scheme: six slices per row
(a signed 7-bit one, then five unsigned bytes, exponent from the row's
largest entry), slice pairs of levels 0..6 summed exactly, the value formed
from two 64-bit integers, the bound E1 + E2 + E3 + E4 doubled. An output
whose interval [ŷ − E, ŷ + E] rounds to one f32 must equal f32 of the
sequential f64 chain matmulOracle computes (forward/oracle.ts:114-125); the
rest are listed. The model is the algorithm, not the kernel: the GPU tests
check the kernel against the FP64 kernel and the oracle.
"""
import math

import numpy as np
import pytest


def slices(X):
    R, K = X.shape
    e = np.zeros(R, np.int64)
    S = np.zeros((6, R, K), np.int64)
    l1, l2 = np.zeros(R), np.zeros(R)
    for r in range(R):
        x = X[r].astype(np.float64)
        mx = np.abs(x).max()
        if mx == 0:
            continue
        e[r] = math.frexp(mx)[1]  # mx < 2^e
        y = np.ldexp(x, 7 - int(e[r]))
        S[0, r] = np.floor(y)
        y = y - S[0, r]
        for i in range(1, 6):
            y = y * 256
            S[i, r] = np.floor(y)
            y = y - S[i, r]
        l1[r] = np.abs(x).sum() * (1 + 2.0 ** -40)
        l2[r] = math.sqrt((x * x).sum()) * (1 + 2.0 ** -40)
    return e, S, l1, l2


def chain(a, b):
    acc = 0.0
    for k in range(a.size):
        acc = acc + float(a[k]) * float(b[k])  # f32 x f32 is exact in f64
    return np.float32(acc)


def decide(A, B):
    K = A.shape[1]
    ea, SA, l1a, l2a = slices(A)
    eb, SB, l1b, l2b = slices(B)
    gamma = (K - 1) * 2.0 ** -53 / (1 - (K - 1) * 2.0 ** -53)
    c2 = K * 65025.0 * sum((11 - L) * 2.0 ** (-14 - 8 * L) for L in range(7, 11))
    Q = np.zeros((7,) + (A.shape[0], B.shape[0]), np.int64)
    for i in range(6):
        for j in range(min(6, 7 - i)):
            Q[i + j] += SA[i] @ SB[j].T
    out = {}
    for m in range(A.shape[0]):
        for n in range(B.shape[0]):
            q = [int(v) for v in Q[:, m, n]]
            hi = (q[0] * 256 + q[1]) * 256 + q[2]
            lo = ((q[3] * 256 + q[4]) * 256 + q[5]) * 256 + q[6]
            assert abs(lo) < 2 ** 53 and abs(hi) < 2 ** 53
            s = int(ea[m] + eb[n])
            y = math.ldexp(float(hi) * 2.0 ** 32 + float(lo), s - 62)
            e1 = math.ldexp(l1b[n], int(ea[m]) - 47) + math.ldexp(l1a[m], int(eb[n]) - 47) + math.ldexp(K, s - 94)
            err = 2 * (e1 + math.ldexp(c2, s) + abs(y) * 2.0 ** -53 + gamma * l2a[m] * l2b[n]) + 2.0 ** -1060
            lo_f, hi_f = np.float32(y - err), np.float32(y + err)
            out[m, n] = lo_f if lo_f.view(np.uint32) == hi_f.view(np.uint32) else None
    return out


@pytest.mark.parametrize("K,seed,relu,spread,scale", [(128, 1, False, 0.0, 1.0), (384, 2, True, 0.0, 1.0),
                                                       (128, 3, False, 12.0, 1e-3), (384, 4, True, 6.0, 30.0)])
def test_settled_outputs_equal_the_chain(K, seed, relu, spread, scale):
    rng = np.random.default_rng(seed)
    A = rng.standard_normal((24, K)) * scale
    if spread:  # entries spread over e^±spread within a row
        A *= np.exp(rng.uniform(-spread, spread, A.shape))
    if relu:
        A = np.maximum(A, 0)
    A = A.astype(np.float32)
    A[3] = 0.0  # an all-zero row
    B = (rng.standard_normal((32, K)) * 0.09).astype(np.float32)
    out = decide(A, B)
    listed = 0
    for (m, n), v in out.items():
        if v is None:
            listed += 1
            continue
        assert v.view(np.uint32) == chain(A[m], B[n]).view(np.uint32), (m, n)
    assert listed <= 0.05 * len(out)
