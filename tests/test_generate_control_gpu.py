"""Cancellation, shutdown and hooks of the generate loop (engine_gen_hooks_t,
reference src/engine/engine.h:96-120; poll sites engine.c:406-470; tests
modelled on tests/test_engine_gpu.c:651-830): poll -> hook -> re-poll at each
prefill chunk, before the seed step and before each decode step."""
import threading
import time

import numpy as np
import pytest

from mlxd_b200 import cuda

pytestmark = pytest.mark.gpu

KW = dict(hidden=256, layers=2, n_heads=4, n_kv_heads=2, head_dim=64, inter=512, vocab=1024,
          max_pos=256)


@pytest.fixture(scope="module")
def model():
    cuda.init(0)
    cfg = cuda.synth_config(**KW)
    m = cuda.Model(cfg, cuda.synth_host_tensors(cfg, seed=2))
    yield m
    m.close()


PROMPT = cuda.synth_prompt(40, KW["vocab"], seed=3)


class Recorder:
    def __init__(self, ctl_kw=None):
        self.events = []
        self.cancel_at = None
        self.ctl = cuda.gen_control(on_prefill_chunk=self.prefill, on_decode_step=self.step,
                                    on_before_seed=self.seed)

    def cancel(self):
        self.ctl.flags[1].value = 1

    def prefill(self, pos, n):
        self.events.append(("prefill", pos, n))
        if self.cancel_at == ("prefill", pos):
            self.cancel()

    def seed(self):
        self.events.append(("seed",))

    def step(self, s):
        self.events.append(("step", s))
        if self.cancel_at == ("step", s):
            self.cancel()


def test_hook_order_on_a_full_request(model):
    r = Recorder()
    toks, _, _ = model.generate(PROMPT, 6, chunk=8, control=r.ctl)
    assert len(toks) == 6 and r.ctl.stopped == 0
    pre = [(e[1], e[2]) for e in r.events if e[0] == "prefill"]
    assert pre == [(0, 8), (8, 8), (16, 8), (24, 8), (32, 7)]   # prompt[:-1] in chunks
    rest = [e for e in r.events if e[0] != "prefill"]
    assert rest == [("seed",)] + [("step", s) for s in range(6)]
    ref, _, _ = model.generate(PROMPT, 6, chunk=8)
    assert np.array_equal(toks, ref)


def test_cancel_in_prefill_hook(model):
    r = Recorder()
    r.cancel_at = ("prefill", 16)
    toks, _, _ = model.generate(PROMPT, 6, chunk=8, control=r.ctl)
    assert len(toks) == 0 and r.ctl.stopped == 1
    assert [e for e in r.events] == [("prefill", 0, 8), ("prefill", 8, 8), ("prefill", 16, 8)]


def test_cancel_in_decode_hook_keeps_the_earlier_tokens(model):
    ref, _, _ = model.generate(PROMPT, 12, chunk=8)
    r = Recorder()
    r.cancel_at = ("step", 5)
    toks, _, _ = model.generate(PROMPT, 12, chunk=8, control=r.ctl)
    assert r.ctl.stopped == 1
    assert np.array_equal(toks, ref[:5])
    assert [e for e in r.events if e[0] == "step"] == [("step", s) for s in range(6)]
    # the model serves the next request normally
    again, _, _ = model.generate(PROMPT, 12, chunk=8)
    assert np.array_equal(again, ref)


def test_shutdown_before_the_call_runs_no_hook(model):
    r = Recorder()
    r.ctl.flags[0].value = 1
    toks, _, _ = model.generate(PROMPT, 6, chunk=8, control=r.ctl)
    assert len(toks) == 0 and r.ctl.stopped == 1 and r.events == []


def test_cancel_while_a_hook_blocks_is_seen_by_the_re_poll():
    """A hook blocks (as a test barrier); another thread sets the cancel flag
    and releases it; the re-poll after the hook ends the request before any
    more work, within the drain bound of 2000 ms."""
    cuda.init(0)
    cfg = cuda.synth_config(**KW)
    m = cuda.Model(cfg, cuda.synth_host_tensors(cfg, seed=2))
    entered, release = threading.Event(), threading.Event()
    seen = []

    def step(s):
        seen.append(s)
        if s == 3:
            entered.set()
            release.wait(30)

    ctl = cuda.gen_control(on_decode_step=step)
    out = {}

    def run():
        out["toks"] = m.generate(PROMPT, 20, chunk=8, control=ctl)[0]
        out["t"] = time.perf_counter()

    th = threading.Thread(target=run)
    th.start()
    assert entered.wait(60)
    ctl.flags[1].value = 1
    t_release = time.perf_counter()
    release.set()
    th.join(60)
    assert not th.is_alive()
    assert ctl.stopped == 1 and len(out["toks"]) == 3 and seen == [0, 1, 2, 3]
    assert (out["t"] - t_release) * 1e3 < 2000
    m.close()
