"""Request server over a pool of denoising contexts.

diffuse-cpp serves one sequence per diffuse_generate call from one caller (its README lists
batching as missing).  Here each request is still one independent sequence -- prompt, number
of tokens to generate, sampler parameters, exactly the arguments of diffuse_generate
(src/diffuse-sampler.cpp:60-370) -- but requests queue up for a pool of contexts: one host
worker thread per context takes the next request in arrival order and runs it to the end.
Contexts on different GPUs run concurrently; contexts of one GPU take turns call by call
(the engine holds a per-device lock around its GEMM calls), overlapping only host work.
Results come back as concurrent.futures.Future objects.

The server owns nothing but threads unless built with from_model(), which loads one model
replica per device and creates the contexts (and frees them on close()).
"""
from __future__ import annotations

import os
import queue
import threading
import time
from concurrent.futures import Future
from dataclasses import dataclass

import numpy as np


@dataclass
class Result:
    tokens: np.ndarray  # the generated ids (n_generate of them; the mask id where none was committed)
    queue_s: float      # seconds between submit() and the start of the generation
    run_s: float        # seconds the generation took on its worker
    worker: int         # index of the context that ran it


class Server:
    """Queue of generation requests served by `contexts` (objects with the Context.generate
    signature), one worker thread each."""

    def __init__(self, contexts):
        if not contexts:
            raise ValueError("a server needs at least one context")
        self._q: queue.Queue = queue.Queue()
        self._lock = threading.Lock()
        self._closed = False
        self._owned = None
        self.n_done = 0
        self.n_tokens = 0
        self._threads = [threading.Thread(target=self._work, args=(i, c), daemon=True, name=f"dfb-worker-{i}")
                         for i, c in enumerate(contexts)]
        for t in self._threads:
            t.start()

    @classmethod
    def from_model(cls, path, devices=(0,), contexts_per_device: int = 1, n_ctx: int = 0):
        """Loads one model replica per device (DIFFUSE_DEVICE selects it at load time) and
        `contexts_per_device` contexts on each."""
        from . import Context, Model  # the package's bindings
        models, contexts = [], []
        saved = os.environ.get("DIFFUSE_DEVICE")
        try:
            for dev in devices:
                os.environ["DIFFUSE_DEVICE"] = str(int(dev))
                m = Model(path)
                models.append(m)
                contexts += [Context(m, n_ctx) for _ in range(contexts_per_device)]
        except BaseException:
            for c in contexts:
                c.close()
            for m in models:
                m.close()
            raise
        finally:
            if saved is None:
                os.environ.pop("DIFFUSE_DEVICE", None)
            else:
                os.environ["DIFFUSE_DEVICE"] = saved
        srv = cls(contexts)
        srv._owned = (models, contexts)
        return srv

    def submit(self, prompt, n_generate: int, params=None) -> Future:
        """Queues one sequence; the future resolves to a Result, or to the generation's error."""
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        if p.ndim != 1 or p.size == 0:
            raise ValueError("prompt must be a non-empty 1-D sequence of token ids")
        if int(n_generate) <= 0:
            raise ValueError("n_generate must be positive")
        fut: Future = Future()
        with self._lock:
            if self._closed:
                raise RuntimeError("server is closed")
            self._q.put((fut, p, int(n_generate), params, time.perf_counter()))
        return fut

    def generate_many(self, requests) -> list:
        """Runs (prompt, n_generate, params) requests; returns their Results in request order
        (raises the first error in that order)."""
        futs = [self.submit(*r) for r in requests]
        return [f.result() for f in futs]

    def _work(self, idx, ctx):
        while True:
            item = self._q.get()
            if item is None:
                return
            fut, prompt, n, params, t_submit = item
            if not fut.set_running_or_notify_cancel():
                continue
            t0 = time.perf_counter()
            try:
                out = ctx.generate(prompt, n, params)
            except BaseException as e:  # the request's error belongs to its future, not the worker
                fut.set_exception(e)
                continue
            t1 = time.perf_counter()
            with self._lock:
                self.n_done += 1
                self.n_tokens += int(n)
            fut.set_result(Result(tokens=out, queue_s=t0 - t_submit, run_s=t1 - t0, worker=idx))

    def close(self, wait: bool = True):
        """Stops taking requests; the queued ones still run.  Frees what from_model() made."""
        with self._lock:
            if self._closed:
                return
            self._closed = True
            for _ in self._threads:
                self._q.put(None)
        if wait:
            for t in self._threads:
                t.join()
            if self._owned:
                models, contexts = self._owned
                for c in contexts:
                    c.close()
                for m in models:
                    m.close()
                self._owned = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
