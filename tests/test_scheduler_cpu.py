"""Continuous-batching scheduler logic on CPU, against a fake engine with the
NativeEngine surface: admission into free slots, slot compaction, per-request
stop on EOS (from min_new_frames on, frame not emitted) or frame budget,
per-frame streaming, capacity checks and independence of the slot a request
runs in (its random stream is fixed, not its slot)."""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from soraku_tts_b200.scheduler import ContinuousBatcher, DecodeRequest

Q, EOS = 16, 2049


def code(seed: int, stream: int, frame: int, q: int) -> int:
    """The fake engine's draw: a hash of (seed, stream, frame, q); q0 of a
    frame listed in the seed's EOS frames is EOS when allowed."""
    h = (seed * 1000003 + stream * 7919 + frame * 104729 + q * 31) & 0x7FFFFFFF
    return h % 2048


class FakeEngine:
    def __init__(self, *, max_requests, rows_per_request, max_len, max_frames, max_prefill, eos_frames=None,
                 page_size=64, kv_pages=0, **kw):
        self.n = max_requests
        self.max_frames = max_frames
        self.max_len = max_len
        self.page_size = page_size
        self.max_pages = -(-max_len // page_size)
        self.shared = kv_pages > 0
        own = [[r * self.max_pages + p for p in range(self.max_pages)] for r in range(2 * max_requests)]
        self.pt = [[-1] * self.max_pages for _ in range(2 * max_requests)] if self.shared else own
        self.eos_frames = eos_frames or {}
        self.st = [dict(seed=0, min=0, frame=0, done=0, stream=i, pos=0) for i in range(max_requests)]
        self.hist = np.zeros((max_requests, max_frames, Q), np.int64)
        self.graph = None
        self.prefill_batch = kw.get("prefill_batch", 1)
        self.kw = kw
        self.log = []

    def set_sampling(self, j, *, seed, min_new_frames, eos_rule, **kw):
        assert eos_rule == 1
        self.st[j].update(seed=seed, min=min_new_frames)

    def set_rng_stream(self, j, stream):
        self.st[j]["stream"] = stream

    def map_pages(self, row, first, pages):
        assert self.shared
        self.pt[row][first:first + len(pages)] = list(pages)

    def _check_pages(self, row, n):
        need = -(-n // self.page_size)
        assert all(p >= 0 for p in self.pt[row][:need]), f"row {row}: positions < {n} not mapped"

    def _check_unique(self, n_active):
        used = [p for row in self.pt[:2 * n_active] for p in row if p >= 0]
        assert len(used) == len(set(used)), "a page is mapped to two rows"

    def prefill(self, j, ids, uncond, prompt, speaker):
        n_prompt = 0 if prompt is None else torch.as_tensor(prompt).numel() // Q
        lc = torch.as_tensor(ids).shape[1] + 1 + n_prompt
        lu = torch.as_tensor(uncond).numel() + 1 + n_prompt
        self._check_pages(2 * j, lc)
        self._check_pages(2 * j + 1, lu)
        self.st[j].update(frame=0, done=0, pos=lc, upos=lu)
        self.log.append(("prefill", j))

    def prefill_many(self, js, conds, uncs, prompts):
        assert len(js) <= self.prefill_batch
        for j, c, u, p in zip(js, conds, uncs, prompts):
            self.prefill(j, c, u, p, None)

    def capture(self, n, fpg):
        self.graph = (n, fpg)
        self.log.append(("capture", n, fpg))

    def step(self, mask_eos_q0=True):
        n, fpg = self.graph
        self._check_unique(n)
        for j in range(n):
            s = self.st[j]
            self._check_pages(2 * j, s["pos"] + fpg)
            self._check_pages(2 * j + 1, s["upos"] + fpg)
            for _ in range(fpg):
                f = s["frame"]
                assert f < self.max_frames and s["pos"] < self.max_len, "capacity exceeded"
                row = [code(s["seed"], s["stream"], f, q) for q in range(Q)]
                if f >= s["min"] and f in self.eos_frames.get(s["seed"], ()):
                    row[0] = EOS
                    s["done"] = 1
                self.hist[j, f] = row
                s["frame"] += 1
                s["pos"] += 1
                s["upos"] += 1

    def status(self, n):
        return [s["frame"] for s in self.st[:n]], [s["done"] for s in self.st[:n]]

    def read_codes(self, j, first, n):
        return torch.from_numpy(self.hist[j, first:first + n].copy())

    def move_request(self, dst, src):
        self.st[dst] = dict(self.st[src])
        self.hist[dst] = self.hist[src]
        for b in range(2):
            self.pt[2 * dst + b], self.pt[2 * src + b] = self.pt[2 * src + b], self.pt[2 * dst + b]
        self.log.append(("move", dst, src))

    def close(self):
        pass


def make(slots=3, fpg=2, eos_frames=None, max_frames=64, max_len=256, kv_pages=None, page_size=64):
    model = SimpleNamespace(config=SimpleNamespace(num_codebooks=Q, audio_eos_id=EOS))
    eng = {}

    def factory(**kw):
        eng["e"] = FakeEngine(eos_frames=eos_frames, **kw)
        return eng["e"]

    b = ContinuousBatcher(model, slots=slots, max_len=max_len, max_frames=max_frames, frames_per_graph=fpg,
                          kv_pages=kv_pages, page_size=page_size, engine_factory=factory)
    return b, eng["e"]


def expected(seed, max_new, min_new, eos_frames):
    rows = []
    for f in range(max_new):
        if f >= min_new and f in eos_frames.get(seed, ()):
            return np.array(rows, np.int64).reshape(-1, Q), "eos"
        rows.append([code(seed, 0, f, q) for q in range(Q)])
    return np.array(rows, np.int64).reshape(-1, Q), "max_frames"


def test_ragged_requests_join_and_leave_with_compaction():
    eos_frames = {105: {3}, 107: {1, 6}, 108: {0}}  # 107: EOS at 1 is masked by min_new_frames=2
    b, e = make(slots=3, fpg=2, eos_frames=eos_frames)
    budgets = [5, 9, 2, 7, 1, 4, 8, 3, 0]
    mins = [0, 0, 0, 0, 0, 2, 2, 0, 0]
    streamed = {}
    for i, (m, mn) in enumerate(zip(budgets, mins)):
        b.submit(DecodeRequest(rid=f"r{i}", input_ids=np.full((1, 3 + i), 7, np.int64),
                               prompt_codes=np.zeros((2 + i, Q), np.int64), max_new_frames=m, min_new_frames=mn,
                               seed=100 + i, on_frame=lambda rid, c: streamed.setdefault(rid, []).append(c)))
    out = b.run()
    assert sorted(out) == sorted(f"r{i}" for i in range(len(budgets)))
    for i, (m, mn) in enumerate(zip(budgets, mins)):
        want, why = expected(100 + i, m, mn, eos_frames)
        got = out[f"r{i}"]
        np.testing.assert_array_equal(got, want)
        assert b.stop_reason[f"r{i}"] == why
        if len(want):
            np.testing.assert_array_equal(np.stack(streamed[f"r{i}"]), want)
        else:
            assert f"r{i}" not in streamed
    assert b.stats["moves"] > 0  # a finished slot below an active one was compacted
    assert b.active() == 0 and b.pending() == 0
    # the graph always covered a contiguous prefix of the slots
    assert all(n <= 3 for kind, *rest in e.log if kind == "capture" for n in rest[:1])


def test_slot_does_not_change_a_request():
    """The same request decoded alone and inside a busy batch: same codes."""
    alone, _ = make(slots=1, fpg=3)
    alone.submit(DecodeRequest(rid="x", input_ids=np.ones((1, 4), np.int64), max_new_frames=10, seed=42))
    a = alone.run()["x"]
    busy, _ = make(slots=4, fpg=3)
    for i in range(5):
        busy.submit(DecodeRequest(rid=i, input_ids=np.ones((1, 4), np.int64), max_new_frames=2 + i, seed=i))
    busy.submit(DecodeRequest(rid="x", input_ids=np.ones((1, 4), np.int64), max_new_frames=10, seed=42))
    np.testing.assert_array_equal(busy.run()["x"], a)


def test_capacity_and_duplicate_checks():
    b, _ = make(slots=2, fpg=4, max_frames=16, max_len=64)
    with pytest.raises(ValueError):
        b.submit(DecodeRequest(rid=0, input_ids=np.ones((1, 4), np.int64), max_new_frames=13))  # 13 + 4 > 16
    with pytest.raises(ValueError):
        b.submit(DecodeRequest(rid=1, input_ids=np.ones((1, 50), np.int64), max_new_frames=10))  # 51 + 10 + 4 > 64
    with pytest.raises(ValueError):
        b.submit(DecodeRequest(rid=2, input_ids=np.ones((4,), np.int64)))  # not [1, L]
    b.submit(DecodeRequest(rid=3, input_ids=np.ones((1, 4), np.int64), max_new_frames=12))
    with pytest.raises(ValueError):
        b.submit(DecodeRequest(rid=3, input_ids=np.ones((1, 4), np.int64), max_new_frames=2))
    out = b.run()
    assert out[3].shape == (12, Q)


def test_shared_kv_pool_admits_by_free_pages():
    """A pool too small for every slot's full reservation: requests wait for
    pages in arrival order, no page is ever mapped to two rows, every page
    returns to the pool, and the codes are those of the own-pages engine."""
    reqs = [(i, 3 + 5 * (i % 3), 4 + 3 * (i % 4)) for i in range(8)]  # (rid, text length, frames)

    def submit_all(b):
        for rid, L, m in reqs:
            b.submit(DecodeRequest(rid=rid, input_ids=np.ones((1, L), np.int64),
                                   prompt_codes=np.zeros((6, Q), np.int64), max_new_frames=m, seed=rid))

    own, _ = make(slots=4, fpg=2, max_len=128, page_size=8)
    submit_all(own)
    want = own.run()
    pooled, e = make(slots=4, fpg=2, max_len=128, page_size=8, kv_pages=14)
    submit_all(pooled)
    got = pooled.run()
    for rid, _, _ in reqs:
        np.testing.assert_array_equal(got[rid], want[rid])
    assert pooled.pool.available() == 14
    assert all(p == -1 for row in e.pt for p in row)
    with pytest.raises(ValueError):  # can never fit the pool
        pooled.submit(DecodeRequest(rid="big", input_ids=np.ones((1, 60), np.int64), max_new_frames=50))
