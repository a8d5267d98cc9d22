"""Request server (diffuse-cpp_b200/serve.py): queueing, per-request parameters, error
routing and worker concurrency with stand-in contexts on the CPU; on a B200, several
contexts of one device serving concurrent requests give the same tokens as one context
running them one after another."""
import threading
import time

import numpy as np
import pytest

from conftest import MINI_LLADA


class FakeContext:
    """Context stand-in: tokens = prompt[0] * 1000 + position + n_steps (so the sampler
    parameters reach it), optional delay, error on a marked prompt."""

    def __init__(self, delay=0.0):
        self.delay = delay
        self.calls = []
        self.active = 0
        self.max_active = 0
        self._lock = threading.Lock()

    def generate(self, prompt, n, params=None):
        with self._lock:
            self.calls.append((int(prompt[0]), n, getattr(params, "n_steps", None)))
        if int(prompt[0]) < 0:
            raise RuntimeError(f"bad prompt {int(prompt[0])}")
        time.sleep(self.delay)
        steps = getattr(params, "n_steps", 0)
        return np.array([int(prompt[0]) * 1000 + j + steps for j in range(n)], np.int32)


def test_requests_complete_in_order_with_their_parameters(pkg):
    ctxs = [FakeContext(), FakeContext()]
    with pkg.serve.Server(ctxs) as srv:
        reqs = [(np.array([i, 5], np.int32), 3 + i % 2, pkg.SamplerParams(n_steps=4 + i)) for i in range(10)]
        res = srv.generate_many(reqs)
    for i, r in enumerate(res):
        assert r.tokens.tolist() == [i * 1000 + j + 4 + i for j in range(3 + i % 2)]
        assert r.worker in (0, 1) and r.run_s >= 0 and r.queue_s >= 0
    assert srv.n_done == 10 and srv.n_tokens == sum(3 + i % 2 for i in range(10))
    assert sorted(c[0] for ctx in ctxs for c in ctx.calls) == list(range(10))


def test_errors_reach_their_own_future(pkg):
    with pkg.serve.Server([FakeContext()]) as srv:
        good = srv.submit([7], 2)
        bad = srv.submit([-1], 2)
        after = srv.submit([8], 2)
        assert good.result().tokens.tolist() == [7000, 7001]
        with pytest.raises(RuntimeError, match="bad prompt -1"):
            bad.result()
        assert after.result().tokens.tolist() == [8000, 8001]


def test_workers_run_concurrently_and_close_drains(pkg):
    ctxs = [FakeContext(delay=0.2) for _ in range(4)]
    srv = pkg.serve.Server(ctxs)
    t0 = time.perf_counter()
    futs = [srv.submit([i], 1) for i in range(8)]
    srv.close()  # queued requests still run
    assert all(f.done() for f in futs)
    wall = time.perf_counter() - t0
    assert wall < 0.8 * 8 * 0.2  # 4 workers: about two rounds of 0.2 s, not eight
    with pytest.raises(RuntimeError, match="closed"):
        srv.submit([1], 1)


def test_bad_requests_are_rejected(pkg):
    with pkg.serve.Server([FakeContext()]) as srv:
        with pytest.raises(ValueError):
            srv.submit([], 4)
        with pytest.raises(ValueError):
            srv.submit([1, 2], 0)
    with pytest.raises(ValueError):
        pkg.serve.Server([])


@pytest.mark.gpu
def test_concurrent_contexts_match_sequential(pkg, model_dir):
    path = pkg.synth_model(model_dir / "serve_llada.gguf", MINI_LLADA, "q4_k_m", seed=21, n_layer=2)
    rng = np.random.default_rng(3)
    reqs = [(rng.integers(0, MINI_LLADA["mask_token_id"] - 1, 12 + 4 * i).astype(np.int32), 16,
             pkg.SamplerParams(n_steps=4, remasking=pkg.LOW_CONFIDENCE if i % 2 else pkg.ENTROPY_EXIT, use_cache=1))
            for i in range(6)]
    model = pkg.Model(path)
    ctx = pkg.Context(model, 64)
    expect = [ctx.generate(p, n, prm) for p, n, prm in reqs]
    ctx.close()
    model.close()
    with pkg.serve.Server.from_model(path, devices=(0,), contexts_per_device=3, n_ctx=64) as srv:
        got = srv.generate_many(reqs)
    for e, g in zip(expect, got):
        assert np.array_equal(e, g.tokens)
