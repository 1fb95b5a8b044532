"""learnFromExperience (packages/krystal/src/host/learn.ts:280-512) with the
gradients from the CUDA backend, for a whole batch of frames at once.

The reference differentiates frame after frame through its GradientSource
(host/gradients.ts:15-24) and updates its own Float32Arrays. Here the split is:

* device (the C ABI): the backward of every frame of a packed batch
  (``kc_backward_batch_device``), each frame's readings for the update — its
  question and bank counts, the critic's baseline, its value loss and report
  terms (``kc_learn_frame_stats``) — and the batch gradients the update
  applies, Σ_f step_f·dSelectorW_f, Σ step_f·dPool_f, Σ dValueWv_f
  (``kc_learn_accumulate``);
* host: the scalar half in the reference's order (which frames count, the
  advantages, their batch mean and deviation, each frame's clipped step;
  learn.ts:318-470), the update of the host's arrays, the parameter-health
  rollback (:479-494), and telling the backend what moved (``sync`` with
  ``WeightChanges``, :495-505).

Several GPUs (one process each, frames split into contiguous shards in rank
order): the per-frame readings are gathered so that every rank computes the
same steps in the same frame order, and the per-rank gradient sums are added
by one all-reduce (NCCL over NVLink on GPUs) before every rank applies the
same update.

On a CUDA backend (``BatchLearner``) the scalar half and the update run on
the device too (``kc_learn_plan``, ``kc_learn_apply``), with token-table
unfreezing (learn.ts:298-299, scatterEmbeddings :242-263). ``plan_update``
and ``apply_update`` below are the same arithmetic on the host: the
reference form the device plan is checked against, and the host half for
gradient sources without a device.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Callable, Sequence

import numpy as np

from . import abi
from .backend import CudaBrainBackend, WeightChanges
from .frame import FrameBatch, pack_host_frame
from .model import BrainForwardWeights
from .session import selection_mask

NO_TARGET = abi.KC_NO_TARGET
NEG_INF = np.float32(-1e30)
STATS = abi.KC_LEARN_STATS  # questions, bank, baseline, loss, entropy total/rows, confidence total/rows


@dataclass
class LearnOptions:
    """LearnOptions (learn.ts:61-139) with the reference's defaults (:292-299)."""
    learning_rate: float = 0.05
    policy_scale: float = 1.0
    advantage_clip: float = 3.0
    max_parameter_abs: float = math.inf
    unfreeze_pool: bool = False
    unfreeze_tokens: bool = False
    token_rate: float = 0.1


@dataclass
class HostExperience:
    """HostExperience (learn.ts:41-59): the records a turn saw, the record each
    question chose (a slot, or -1), what it was worth, the grammar it chose under."""
    records: Sequence
    reward: float | None = None
    chosen: Sequence[int] | None = None
    allows: Callable[[int, int], bool] | None = None


@dataclass
class LearnReport:
    """LearnReport (learn.ts:141-164), as filled at :470-511."""
    frames_seen: int
    mean_advantage: float
    mean_value_loss: float
    reinforced: int
    discouraged: int
    mean_entropy: float
    mean_confidence: float
    update_applied: bool
    rejected: str | None = None
    health: dict = field(default_factory=dict)


@dataclass
class UpdatePlan:
    step: np.ndarray          # [F] f64: the weight each frame's actor gradient enters the update with
    value_weight: np.ndarray  # [F] f64: 1 for a frame the critic learns from
    seen: int
    actor_moved: bool
    reinforced: int
    discouraged: int
    mean_advantage: float
    mean_value_loss: float
    mean_entropy: float
    mean_confidence: float


def _running_total(x: np.ndarray) -> float:
    """The loop's `total += x[i]` from 0.0, in order: the last running sum
    (np.cumsum adds sequentially; np.sum would pair terms)."""
    return float(np.cumsum(np.concatenate(([0.0], x)))[-1])


def plan_update(stats: np.ndarray, rewards: np.ndarray, answered: np.ndarray, options: LearnOptions) -> UpdatePlan:
    """The scalar half of learnFromExperience over a batch, in batch order.

    stats: [F, 8] per-frame readings (kc_learn_frame_stats); rewards: [F]
    (NaN = no reward: the experience is skipped, learn.ts:320); answered: [F]
    whether any question had a target (:325-334). Vectorised, with every sum
    taken in frame order as the reference's loop takes it."""
    stats = np.asarray(stats, np.float64)
    rewards = np.asarray(rewards, np.float64)
    F = rewards.size
    step = np.zeros(F, np.float64)
    value_weight = np.zeros(F, np.float64)
    used = np.flatnonzero(~np.isnan(rewards) & (stats[:, 0] != 0) & (stats[:, 1] != 0))
    advantage = rewards[used] - stats[used, 2]
    value_weight[used] = 1.0
    seen = int(used.size)
    adv_total, loss_total = _running_total(advantage), _running_total(stats[used, 3])
    ent_total, ent_rows = _running_total(stats[used, 4]), _running_total(stats[used, 5])
    conf_total, conf_rows = _running_total(stats[used, 6]), _running_total(stats[used, 7])
    pend = np.asarray(answered, bool)[used] & np.isfinite(advantage)
    frames, adv = used[pend], advantage[pend]
    reinforced = discouraged = 0
    actor_moved = False
    if adv.size:
        n = adv.size
        mean = _running_total(adv) / n
        d = adv - mean
        var = _running_total(d * d) / n  # (a - mean) ** 2: a square, as the reference's pow(x, 2) is
        deviation = math.sqrt(var)
        if deviation > 1e-6:  # a batch where everything went equally well pushes nothing (:447-451)
            actor_moved = True
            clip = options.advantage_clip
            st = np.minimum(clip, np.maximum(-clip, (adv - mean) / deviation))
            step[frames] = (options.learning_rate * options.policy_scale * st) / n
            reinforced = int((st > 0).sum())
            discouraged = int((st < 0).sum())
    return UpdatePlan(step, value_weight, seen, actor_moved, reinforced, discouraged,
                      adv_total / seen if seen else 0.0, loss_total / seen if seen else 0.0,
                      ent_total / ent_rows if ent_rows else 0.0, conf_total / conf_rows if conf_rows else 0.0)


def _max_abs(a: np.ndarray) -> float:
    a = np.abs(a.astype(np.float64))
    if not np.all(np.isfinite(a)):
        return math.inf
    return float(a.max()) if a.size else 0.0


def parameter_health(weights: BrainForwardWeights) -> dict:
    """parameterHealth (learn.ts:186-205) without embedding rows (tokens stay frozen)."""
    sel = max(_max_abs(weights.selector.wq), _max_abs(weights.selector.wk))
    h = dict(semantic_embedding_max_abs=0.0, selector_max_abs=sel, value_max_abs=_max_abs(weights.value_head_wv),
             pool_max_abs=_max_abs(weights.pool))
    h["finite"] = all(math.isfinite(v) for v in h.values())
    return h


def apply_update(weights: BrainForwardWeights, sums: np.ndarray, plan: UpdatePlan,
                 options: LearnOptions) -> tuple[WeightChanges | None, str | None, dict]:
    """Apply the batch gradients to the host's arrays (learn.ts:432-470), check
    parameter health and roll back a rejected update (:479-494). Returns what
    the backend must take up (None after a rollback or an empty batch)."""
    h = weights.config.hidden_size
    hh = h * h
    s_wq, s_wk = sums[:hh], sums[hh:2 * hh]
    s_pool, s_dv = sums[2 * hh:2 * hh + 2 * h], sums[2 * hh + 2 * h:2 * hh + 5 * h]
    before = (weights.selector.wq.copy(), weights.selector.wk.copy(), weights.value_head_wv.copy(),
              weights.pool.copy())
    lr = options.learning_rate
    if plan.seen:
        wv = weights.value_head_wv
        wv[:] = (wv.astype(np.float64) - (lr * s_dv) / plan.seen).astype(np.float32)
    if plan.actor_moved:
        for dst, s in ((weights.selector.wq, s_wq), (weights.selector.wk, s_wk)) + (
                ((weights.pool, s_pool),) if options.unfreeze_pool else ()):
            dst[:] = (dst.astype(np.float64) - s).astype(np.float32)
    attempted = parameter_health(weights)
    over = any(attempted[k] > options.max_parameter_abs
               for k in ("semantic_embedding_max_abs", "selector_max_abs", "value_max_abs", "pool_max_abs"))
    rejected = "non-finite" if not attempted["finite"] else "parameter-limit" if over else None
    if rejected:
        for dst, src in zip((weights.selector.wq, weights.selector.wk, weights.value_head_wv, weights.pool), before):
            dst[:] = src
        return None, rejected, parameter_health(weights)
    if not plan.seen:
        return None, None, attempted
    changes = WeightChanges(value_head=True, selector=plan.actor_moved,
                            pool=plan.actor_moved and options.unfreeze_pool)
    return changes, None, attempted


def shard_bounds(frames: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous frame shard of `rank`: frames [start, stop)."""
    return frames * rank // world, frames * (rank + 1) // world


def gather_frame_rows(local: np.ndarray, global_frames: int, group) -> np.ndarray:
    """All ranks' per-frame rows [F_r, C] in global frame order (every rank
    holds the contiguous shard shard_bounds(global_frames, world, rank)).
    NCCL gathers device tensors, other backends host tensors."""
    import torch
    import torch.distributed as dist
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    fmax = -(-global_frames // world)
    pad = np.full((fmax, local.shape[1]), np.nan)
    pad[:local.shape[0]] = local
    dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" else "cpu"
    t = torch.from_numpy(pad).to(dev)
    outs = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(outs, t, group=group)
    parts = []
    for r in range(world):
        a, b = shard_bounds(global_frames, world, r)
        parts.append(outs[r].cpu().numpy()[:b - a])
    return np.concatenate(parts)


def all_reduce_sums(sums, group) -> np.ndarray:
    """Add every rank's gradient sums (f64) and return the total on the host:
    the one gradient exchange of the learn step. `sums` is a torch tensor on
    the collective's device (a CUDA tensor for NCCL)."""
    import torch.distributed as dist
    dist.all_reduce(sums, group=group)
    return sums.cpu().numpy()


def gather_frame_rows_device(local, global_frames: int, group):
    """All ranks' per-frame rows [F_r, C] (a CUDA tensor) in global frame
    order, on the device: one NCCL all-gather, no host copy."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    fmax = -(-global_frames // world)
    pad = torch.zeros((fmax, local.shape[1]), dtype=local.dtype, device=local.device)
    pad[:local.shape[0]] = local
    out = torch.empty((world * fmax, local.shape[1]), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, pad, group=group)
    keep = torch.cat([torch.arange(r * fmax, r * fmax + (b - a), device=local.device)
                      for r, (a, b) in ((r, shard_bounds(global_frames, world, r)) for r in range(world))])
    return out.index_select(0, keep)


class BatchLearner:
    """The learn step over device-resident batches for one backend (one GPU).

    The backward, the per-frame readings, the update plan, the gradient sums,
    the update of the device's weight page with its health check and rollback
    all run on the device in stream order (``kc_learn_plan``,
    ``kc_learn_accumulate[_rows]``, ``kc_learn_apply``); the host's arrays are
    then read back from the page. ``group``: a torch.distributed process
    group for several GPUs, every rank holding the contiguous shard
    ``shard_bounds(global_frames, world, rank)``; the per-frame rows are
    all-gathered and the gradient sums all-reduced on the device, so that
    every rank plans and applies the same update.
    """

    def __init__(self, backend: CudaBrainBackend, weights: BrainForwardWeights, group=None):
        import torch
        self.torch = torch
        self.be = backend
        self.weights = weights
        self.group = group
        cfg = backend.config
        h = cfg.hidden_size
        self.dev = torch.device("cuda", backend.device)
        self.sums = torch.zeros(2 * h * h + 5 * h, dtype=torch.float64, device=self.dev)
        self.stats = torch.zeros(0, dtype=torch.float64, device=self.dev)
        self.report = torch.zeros(abi.KC_LEARN_REPORT, dtype=torch.float64, device=self.dev)
        self.table_rows = cfg.token_space + cfg.field_space
        self.stream = torch.cuda.Stream(device=self.dev)
        self.rows_buf = None  # [table rows * H + table rows] f64: row sums, then touched flags
        self._pinned = {}

    def _to_device(self, name: str, a: np.ndarray):
        """a host array through a reused pinned buffer, copied without waiting."""
        torch = self.torch
        t = self._pinned.get(name)
        if t is None or t.numel() < a.size:
            t = torch.empty(max(a.size, 1), dtype=torch.float64).pin_memory()
            self._pinned[name] = t
        t[:a.size] = torch.from_numpy(a)
        return t[:a.size].to(self.dev, non_blocking=True)

    def _options(self, o: LearnOptions) -> abi.KcLearnOptions:
        return abi.KcLearnOptions(o.learning_rate, o.policy_scale, o.advantage_clip, o.max_parameter_abs,
                                  o.token_rate, int(o.unfreeze_pool), int(o.unfreeze_tokens))

    def step(self, frames: int, records: int, rec_off: int, token_ids: int, field_roles: int, schema_ids: int,
             band_ids: int, rewards: np.ndarray, answered: np.ndarray, targets: int | None = None,
             selection: int | None = None, schema_allow: int | None = None, band_allow: int | None = None,
             options: LearnOptions = LearnOptions(), global_frames: int | None = None) -> LearnReport:
        """One update from a device-resident batch (raw device pointers as for
        kc_backward_batch_device). rewards [frames] f64 (NaN = none), answered
        [frames] bool, host arrays for this rank's frames. The library runs
        the step on a torch stream, and every torch operation of the step
        (copies, the row table, the collectives) is queued on it, in order
        with the library's kernels; the library's stream is restored after."""
        torch = self.torch
        # a stream torch owns (never destroyed under its tensors): the caller's
        # current one, or the learner's own when that is the default stream
        cur = torch.cuda.current_stream(self.dev)
        run = cur if cur.cuda_stream else self.stream
        prev = self.be.stream_ptr()
        self.be.set_stream(run.cuda_stream)
        try:
            with torch.cuda.stream(run):
                return self._step(frames, records, rec_off, token_ids, field_roles, schema_ids, band_ids, rewards,
                                  answered, targets, selection, schema_allow, band_allow, options, global_frames)
        finally:
            self.be.set_stream(prev)

    def _step(self, frames, records, rec_off, token_ids, field_roles, schema_ids, band_ids, rewards, answered,
              targets, selection, schema_allow, band_allow, options, global_frames) -> LearnReport:
        torch = self.torch
        rewards = np.ascontiguousarray(rewards, np.float64)
        valence = self._to_device("rewards", rewards)
        flags = self._to_device("answered", np.asarray(answered, np.float64))
        self.be.backward_batch_device(frames, records, rec_off, token_ids, field_roles, schema_ids, band_ids,
                                      selection, targets, valence.data_ptr(), schema_allow, band_allow)
        if self.stats.numel() < frames * STATS:
            self.stats = torch.empty(frames * STATS, dtype=torch.float64, device=self.dev)
        self.be.learn_frame_stats(targets, self.stats.data_ptr())
        local = torch.cat([self.stats[:frames * STATS].view(frames, STATS), valence.view(frames, 1),
                           flags.view(frames, 1)], 1).contiguous()
        lo = 0
        rows = local
        if self.group is not None:
            import torch.distributed as dist
            g = global_frames if global_frames is not None else frames
            rows = gather_frame_rows_device(local, g, self.group)
            lo, _ = shard_bounds(g, dist.get_world_size(self.group), dist.get_rank(self.group))
        n = rows.shape[0]
        plan = torch.empty((3, max(n, 1)), dtype=torch.float64, device=self.dev)  # step, value weight, pending
        step, vw, pend = plan[0], plan[1], plan[2]
        opts = self._options(options)
        self.be.learn_plan(rows.data_ptr(), n, opts, step.data_ptr(), vw.data_ptr(), pend.data_ptr(),
                           self.report.data_ptr())
        self.be.learn_accumulate(step[lo:].data_ptr(), vw[lo:].data_ptr(), self.sums.data_ptr())
        row_sums = touched = None
        h = self.be.config.hidden_size
        if options.unfreeze_tokens:
            if self.rows_buf is None:
                self.rows_buf = torch.zeros(self.table_rows * (h + 1), dtype=torch.float64, device=self.dev)
            self.rows_buf.zero_()
            row_sums, touched = self.rows_buf[:self.table_rows * h], self.rows_buf[self.table_rows * h:]
            self.be.learn_accumulate_rows(token_ids, field_roles, step[lo:].data_ptr(), pend[lo:].data_ptr(),
                                          row_sums.data_ptr(), touched.data_ptr())
        if self.group is not None:
            import torch.distributed as dist
            dist.all_reduce(self.sums, group=self.group)
            if row_sums is not None:
                dist.all_reduce(self.rows_buf, group=self.group)
        result = self.be.learn_apply(self.sums.data_ptr(), row_sums.data_ptr() if row_sums is not None else None,
                                     touched.data_ptr() if touched is not None else None,
                                     self.report.data_ptr(), opts)
        report = result[10:]
        self._read_back(options, moved=report[1] != 0.0 and result[0] != 0.0)
        rejected = {0: None, 1: "non-finite", 2: "parameter-limit"}[int(result[1])]
        health = dict(semantic_embedding_max_abs=float(result[3]), selector_max_abs=float(result[4]),
                      value_max_abs=float(result[5]), pool_max_abs=float(result[6]), finite=bool(result[2]))
        return LearnReport(int(report[0]), float(report[4]), float(report[5]), int(report[2]), int(report[3]),
                           float(report[6]), float(report[7]), bool(result[0]), rejected, health)

    def _read_back(self, options: LearnOptions, moved: bool) -> None:
        """The host's arrays as the device page left them."""
        w, lay = self.weights, self.weights.layout
        self.be.copy_weights(lay.selector_wq, w.page[lay.selector_wq:lay.total])  # selector, decision and value heads
        self.be.copy_weights(lay.pool, w.pool)
        if options.unfreeze_tokens and moved:
            h = self.be.config.hidden_size
            self.be.copy_weights(lay.embeddings, w.embeddings[:self.table_rows * h])


def experience_batch(experiences: Sequence[HostExperience]) -> tuple[FrameBatch, np.ndarray, np.ndarray,
                                                                    np.ndarray, np.ndarray]:
    """Pack the experiences that carry a reward and records (learn.ts:319-320)
    into a batch: the batch, per-frame rewards and answered flags, the
    selection masks laid out like the batch's p, and per-question targets
    (the chosen slot's bank row, learn.ts:325-334)."""
    frames, rewards, answered, masks, targets = [], [], [], [], []
    for ex in experiences:
        if ex.reward is None or not len(ex.records):
            continue
        frame = pack_host_frame(ex.records)
        act = frame.active
        q, r = act.query_records.size, act.bank_records.size
        bank = act.bank_records.tolist()
        tg = np.full(q, NO_TARGET, np.uint32)
        for i in range(q):
            slot = ex.chosen[i] if ex.chosen is not None and i < len(ex.chosen) else None
            if slot is None or slot < 0 or slot not in bank:
                continue
            tg[i] = bank.index(slot)
        frames.append(frame.gpu)
        rewards.append(float(ex.reward))
        answered.append(bool((tg != NO_TARGET).any()))
        masks.append(selection_mask(act, ex.allows))
        targets.append(tg)
    counts = np.array([f.schema_ids.size for f in frames], dtype=np.uint64)
    rec_off = np.zeros(len(frames) + 1, dtype=np.uint64)
    np.cumsum(counts, out=rec_off[1:])
    cat = lambda xs, dt: np.concatenate(xs).astype(dt) if xs else np.zeros(0, dt)  # noqa: E731
    batch = FrameBatch(rec_off, cat([f.token_ids for f in frames], np.uint32),
                       cat([f.field_roles for f in frames], np.uint32), cat([f.schema_ids for f in frames], np.uint32),
                       cat([f.band_ids for f in frames], np.uint32))
    return (batch, np.array(rewards, np.float64), np.array(answered, bool), cat(masks, np.float32),
            cat(targets, np.uint32))


def learn_from_experience(experiences: Sequence[HostExperience], weights: BrainForwardWeights,
                          backend: CudaBrainBackend, options: LearnOptions = LearnOptions(),
                          learner: BatchLearner | None = None) -> LearnReport:
    """learnFromExperience (learn.ts:280-512) with the backend as the gradient
    source: one batch backward on the device, the update on the host arrays,
    the backend synced with what moved."""
    import torch
    batch, rewards, answered, masks, targets = experience_batch(experiences)
    if batch.frames == 0:
        return LearnReport(0, 0.0, 0.0, 0, 0, 0.0, 0.0, False, None, parameter_health(weights))
    learner = learner or BatchLearner(backend, weights)
    dev = learner.dev
    as_dev = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int32)).to(dev)  # noqa: E731
    tok, role, sch, band = (as_dev(batch.token_ids), as_dev(batch.field_roles), as_dev(batch.schema_ids),
                            as_dev(batch.band_ids))
    rec_off = torch.from_numpy(batch.rec_off.astype(np.int64)).to(dev)
    sel = torch.from_numpy(np.ascontiguousarray(masks, np.float32)).to(dev) if masks.size else None
    tg = as_dev(targets) if targets.size else None
    return learner.step(batch.frames, batch.records, rec_off.data_ptr(), tok.data_ptr(), role.data_ptr(),
                        sch.data_ptr(), band.data_ptr(), rewards, answered, tg.data_ptr() if tg is not None else None,
                        sel.data_ptr() if sel is not None else None, options=options)
