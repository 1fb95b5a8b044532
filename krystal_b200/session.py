"""BrainSession over the CUDA backend: records in, one choice per question out.

Mirrors packages/krystal/src/host/session.ts (``BrainSession`` :106-255,
``consider``/``think``/``choose`` :128-181, ``HostSelection`` :59-69) with the
selector moved onto the device through the backend's ``select`` — the
optional seam extension; the mask is built by ``selection_mask`` exactly as
the reference builds it (host/learn.ts:215-232), so choosing and learning see
the same grammar. ``snapshot``/``restore`` write and read KRY1 checkpoints
(session.ts:226-249); learning lives in ``krystal_b200.learn``.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Sequence

import numpy as np

from .backend import CudaBrainBackend, EncodedFrame, cuda_backend
from .checkpoint import decode_checkpoint, encode_checkpoint
from .frame import HostFrame, pack_host_frame
from .model import BRAIN_FORWARD_CONFIG, BrainForwardConfig, BrainForwardWeights, create_brain_forward_weights, \
    validate_brain_forward_weights

NEG_INF = np.float32(-1e30)  # forward/oracle.ts:36


def selection_mask(active, allows: Callable[[int, int], bool] | None) -> np.ndarray:
    """selectionMask (host/learn.ts:215-232): [Q,R], NEG_INF where `allows` says no;
    a question nothing admits is left open."""
    q, r = active.query_records.size, active.bank_records.size
    mask = np.zeros(q * r, dtype=np.float32)
    if allows is None:
        return mask
    bank = active.bank_records.tolist()
    for i in range(q):
        admitted = 0
        for j, slot in enumerate(bank):
            if allows(i, slot):
                admitted += 1
            else:
                mask[i * r + j] = NEG_INF
        if not admitted:
            mask[i * r:(i + 1) * r] = 0
    return mask


@dataclass
class HostSelection:
    query: int
    record: int | None
    probability: float
    distribution: np.ndarray


@dataclass
class ThinkResult:
    selections: list[HostSelection]
    frame: HostFrame


class Deliberation:
    """A frame that has been read, waiting to be asked about (session.ts:85-90)."""

    def __init__(self, frame: HostFrame, session: "BrainSession", encoded: EncodedFrame | None):
        self.frame = frame
        self._session = session
        self._encoded = encoded

    def choose(self, allows: Callable[[int, int], bool] | None = None,
               sample: Callable[[int], float] | None = None) -> ThinkResult:
        active = self.frame.active
        q, r = active.query_records.size, active.bank_records.size
        if self._encoded is None:
            return ThinkResult([], self.frame)
        mask = selection_mask(active, allows)
        uniforms = None if sample is None else np.array([sample(i) for i in range(q)], dtype=np.float64)
        sel = self._session.backend.select(self._encoded, mask=mask, uniforms=uniforms, gather=False)
        out = []
        for i in range(q):
            chosen = int(sel.index[i])
            dist = sel.p[i * r:(i + 1) * r].copy()
            ok = chosen < r
            out.append(HostSelection(i, int(active.bank_records[chosen]) if ok else None,
                                     float(dist[chosen]) if ok else 0.0, dist))
        return ThinkResult(out, self.frame)


class BrainSession:
    """session.ts:106-255 with a device backend (the CUDA one by default)."""

    def __init__(self, token_rows, seed: int = 1337, weights: BrainForwardWeights | None = None,
                 config: BrainForwardConfig | None = None,
                 backend: Callable[[BrainForwardConfig, BrainForwardWeights], CudaBrainBackend] | None = None):
        self.config = (config or BRAIN_FORWARD_CONFIG).with_token_rows(token_rows)
        self.weights = weights or create_brain_forward_weights(self.config, seed)
        validate_brain_forward_weights(self.config, self.weights)
        self.backend = (backend or cuda_backend())(self.config, self.weights)

    def consider(self, records: Sequence) -> Deliberation:
        frame = pack_host_frame(records)
        if not frame.active.query_records.size or not frame.active.bank_records.size:
            return Deliberation(frame, self, None)
        return Deliberation(frame, self, self.backend.encode(frame))

    def think(self, records: Sequence, allows=None, sample=None) -> ThinkResult:
        return self.consider(records).choose(allows, sample)

    def learn(self, experiences: Sequence, options=None):
        """session.ts:195-197: one pass over remembered turns (learnFromExperience),
        the backend differentiating and told what moved."""
        from .learn import LearnOptions, learn_from_experience
        return learn_from_experience(experiences, self.weights, self.backend, options or LearnOptions())

    def teach(self, demonstrations: Sequence, options=None):
        """session.ts:205-207: be shown what can be said here (teachFromDemonstration)."""
        from .teach import TeachOptions, teach_from_demonstration
        return teach_from_demonstration(demonstrations, self.weights, self.backend, options or TeachOptions())

    def sync(self, changes=None) -> None:
        self.backend.sync(self.weights, changes)

    def snapshot(self) -> bytes:
        """session.ts:235-237: the weights, their geometry and vocabulary as KRY1."""
        return encode_checkpoint(self.weights, self.config, self.config.token_rows)

    def restore(self, data) -> str | None:
        """session.ts:245-249: take up a checkpoint in place, or say why it does
        not fit. The device page takes the same bytes directly."""
        refusal = decode_checkpoint(data, self.weights, self.config, self.config.token_rows)
        if refusal is None:
            device_refusal = self.backend.load_checkpoint(data)
            if device_refusal is not None:  # the host took it: the device must hold the same weights
                self.backend.sync(self.weights)
        return refusal

    def destroy(self) -> None:
        self.backend.destroy()
