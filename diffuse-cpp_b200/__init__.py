"""Python bindings of the B200 denoising engine (ctypes over the C-ABI).

Mirrors the reference's public API (include/diffuse.h of diffuse-cpp): load a GGUF
model, make a context, run `forward` (diffuse_forward) or `generate`
(diffuse_generate).  Everything computes in lib/libdfb_cuda.so (sm_100a kernels);
there is no CPU fallback: on a machine without a B200 the calls fail with the
engine's error message.

The directory name carries a hyphen, so load it by path::

    spec = importlib.util.spec_from_file_location("diffuse_b200", ".../diffuse-cpp_b200/__init__.py")
"""
from __future__ import annotations

import ctypes as C
import os
import pathlib
from dataclasses import dataclass

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
LIB_DIR = HERE / "lib"

# GGML type ids
F32, F16, Q8_0, Q4_K, Q6_K, BF16 = 0, 1, 8, 12, 14, 30
# remasking / schedule enums of include/diffuse.h
LOW_CONFIDENCE, RANDOM, ENTROPY_EXIT, MASKGIT_PLUS, TOPK_MARGIN = 0, 1, 2, 3, 4
COSINE, LINEAR = 0, 1
# engine tensor roles (include/diffuse_b200.h)
(TOK_EMBD, OUTPUT_NORM, OUTPUT, ATTN_NORM, WQ, WK, WV, WO, BQ, BK, BV, FFN_NORM, GATE, UP, DOWN) = range(15)


class DiffuseError(RuntimeError):
    pass


class SamplerParams(C.Structure):
    """dfb_sampler_params == diffuse_sampler_params field by field (same defaults)."""
    _fields_ = [("n_steps", C.c_int32), ("temperature", C.c_float), ("schedule", C.c_int32),
                ("remasking", C.c_int32), ("seed", C.c_uint32), ("entropy_threshold", C.c_float),
                ("use_cache", C.c_int32), ("cache_refresh", C.c_int32), ("cache_keep_active", C.c_int32)]

    def __init__(self, **kw):
        d = dict(n_steps=32, temperature=0.0, schedule=COSINE, remasking=LOW_CONFIDENCE, seed=42,
                 entropy_threshold=1.5, use_cache=1, cache_refresh=0, cache_keep_active=0)
        d.update(kw)
        super().__init__(**{k: (int(v) if isinstance(v, bool) else v) for k, v in d.items()})


class Trace(C.Structure):
    _fields_ = [("max_steps", C.c_int32), ("steps_run", C.c_int32), ("n_active", C.POINTER(C.c_int32)),
                ("n_unmasked", C.POINTER(C.c_int32)), ("commit_pos", C.POINTER(C.c_int32)),
                ("commit_tok", C.POINTER(C.c_int32)), ("fwd_ms", C.POINTER(C.c_float)),
                ("step_ms", C.POINTER(C.c_float)), ("total_ms", C.c_double)]


class BatchTrace(C.Structure):
    _fields_ = [("max_steps", C.c_int32), ("steps_run", C.c_int32), ("n_active", C.POINTER(C.c_int32)),
                ("n_unmasked", C.POINTER(C.c_int32)), ("fwd_ms", C.POINTER(C.c_float)),
                ("step_ms", C.POINTER(C.c_float)), ("total_ms", C.c_double)]


class SynthSpec(C.Structure):
    _fields_ = [("is_dream", C.c_int32), ("n_vocab", C.c_int32), ("n_embd", C.c_int32), ("n_head", C.c_int32),
                ("n_head_kv", C.c_int32), ("n_layer", C.c_int32), ("n_ff", C.c_int32), ("n_ctx", C.c_int32),
                ("mask_token_id", C.c_int32), ("rope_theta", C.c_float), ("rms_norm_eps", C.c_float),
                ("scheme", C.c_int32), ("with_bias", C.c_int32), ("tied_output", C.c_int32),
                ("seed", C.c_uint64), ("w_std", C.c_float), ("n_threads", C.c_int32)]


SCHEMES = {"f32": 0, "f16": 1, "q8_0": 2, "q4_k_m": 3}

# Architectures of BASELINE.json's configs (LLaDA-8B, Dream-7B).
LLADA_8B = dict(is_dream=0, n_vocab=126464, n_embd=4096, n_head=32, n_head_kv=32, n_layer=32, n_ff=12288,
                n_ctx=4096, mask_token_id=126336, rope_theta=500000.0, rms_norm_eps=1e-5, with_bias=0)
DREAM_7B = dict(is_dream=1, n_vocab=152064, n_embd=3584, n_head=28, n_head_kv=4, n_layer=28, n_ff=18944,
                n_ctx=131072, mask_token_id=151666, rope_theta=1000000.0, rms_norm_eps=1e-6, with_bias=1)

_libs = {}


def _load():
    if _libs:
        return _libs
    cu = LIB_DIR / "libdfb_cuda.so"
    host = LIB_DIR / "libdiffuse.so"
    if not cu.exists() or not host.exists():
        raise DiffuseError(f"native libraries missing in {LIB_DIR}; run `make -C {HERE}` (or __graft_entry__.build())")
    dfb = C.CDLL(str(cu), mode=C.RTLD_GLOBAL)
    dfc = C.CDLL(str(host), mode=C.RTLD_GLOBAL)
    P, I, F = C.c_void_p, C.c_int, C.c_float
    sig = {
        (dfb, "dfb_last_error"): (C.c_char_p, []),
        (dfb, "dfb_device_count"): (I, [C.POINTER(I)]),
        (dfb, "dfb_forward"): (I, [P, P, I, P]),
        (dfb, "dfb_linear"): (I, [P, I, I, P, I, P]),
        (dfb, "dfb_debug_stalled_linear"): (I, [P, I, I, P, I, P, C.c_ulonglong]),
        (dfb, "dfb_gen_begin"): (I, [P, P, I, I, C.POINTER(SamplerParams)]),
        (dfb, "dfb_gen_step"): (I, [P, I, I, I, P, P]),
        (dfb, "dfb_gen_set_uniforms"): (I, [P, P, I]),
        (dfb, "dfb_gen_tokens"): (I, [P, P, I]),
        (dfb, "dfb_gen_commits"): (I, [P, P, P, I]),
        (dfb, "dfb_gen_logits"): (I, [P, I, I, P]),
        (dfb, "dfb_gen_begin_batch"): (I, [P, I, P, P, P, C.POINTER(SamplerParams)]),
        (dfb, "dfb_gen_step_batch"): (I, [P, I, P, I, P, P]),
        (dfb, "dfb_gen_commits_batch"): (I, [P, P, P, P, I]),
        (dfc, "dfc_generate_batch"): (I, [P, P, P, I, I, C.POINTER(SamplerParams), P, P]),
        (dfb, "dfb_ctx_stream"): (I, [P, C.POINTER(P)]),
        (dfc, "dfc_last_error"): (C.c_char_p, []),
        (dfc, "dfc_model_load"): (P, [C.c_char_p, I]),
        (dfc, "dfc_model_load_tp"): (P, [C.c_char_p, I, I, P, I]),
        (dfc, "dfc_model_tp_info"): (I, [P, P, P, P, P]),
        (dfb, "dfb_tp_unique_id"): (I, [P, I]),
        (dfc, "dfc_model_free"): (None, [P]),
        (dfc, "dfc_model_hparams"): (I, [P, P, P]),
        (dfc, "dfc_context_new"): (P, [P, I, I]),
        (dfc, "dfc_context_free"): (None, [P]),
        (dfc, "dfc_context_engine"): (P, [P]),
        (dfc, "dfc_forward"): (I, [P, P, I, P]),
        (dfc, "dfc_generate"): (I, [P, P, I, I, C.POINTER(SamplerParams), P, C.POINTER(Trace)]),
        (dfc, "dfc_quantize_file"): (I, [C.c_char_p, C.c_char_p, C.c_char_p, I]),
        (dfc, "dfc_synth_model"): (I, [C.c_char_p, C.POINTER(SynthSpec)]),
        (dfc, "dfc_quantize_rows"): (I, [I, P, C.c_int64, P]),
        (dfc, "dfc_dequantize_rows"): (I, [I, P, C.c_int64, P]),
        (dfc, "dfc_tokens_to_unmask"): (I, [I, I, I, I]),
    }
    for (lib, name), (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype, fn.argtypes = res, args
    _libs.update(dfb=dfb, dfc=dfc)
    return _libs


def native():
    """(libdfb_cuda, libdiffuse) ctypes handles."""
    L = _load()
    return L["dfb"], L["dfc"]


def _dfb_err():
    return native()[0].dfb_last_error().decode()


def _dfc_err():
    return native()[1].dfc_last_error().decode()


def _ptr(a):
    return a.ctypes.data_as(C.c_void_p)


def device_count() -> int:
    n = C.c_int(0)
    native()[0].dfb_device_count(C.byref(n))
    return n.value


# ── codecs / fixtures (host only, no GPU needed) ──
ROW_BYTES = {F32: (1, 4), F16: (1, 2), BF16: (1, 2), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210)}


def quantize_rows(x: np.ndarray, ggml_type: int) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    blk, sz = ROW_BYTES[ggml_type]
    out = np.zeros(x.size // blk * sz, dtype=np.uint8)
    if native()[1].dfc_quantize_rows(ggml_type, _ptr(x), x.size, _ptr(out)) != 0:
        raise DiffuseError(_dfc_err())
    return out


def dequantize_rows(raw: np.ndarray, ggml_type: int, n: int) -> np.ndarray:
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    out = np.zeros(n, dtype=np.float32)
    if native()[1].dfc_dequantize_rows(ggml_type, _ptr(raw), n, _ptr(out)) != 0:
        raise DiffuseError(_dfc_err())
    return out


def synth_model(path, arch: dict, scheme: str = "q4_k_m", seed: int = 0, w_std: float = 0.02,
                tied_output: bool = False, n_threads: int = 0, **overrides):
    """Write a seeded random-init GGUF (converter metadata, reference quantization policy)."""
    a = dict(arch)
    a.update(overrides)
    spec = SynthSpec(is_dream=a["is_dream"], n_vocab=a["n_vocab"], n_embd=a["n_embd"], n_head=a["n_head"],
                     n_head_kv=a["n_head_kv"], n_layer=a["n_layer"], n_ff=a["n_ff"], n_ctx=a.get("n_ctx", 4096),
                     mask_token_id=a["mask_token_id"], rope_theta=a["rope_theta"], rms_norm_eps=a["rms_norm_eps"],
                     scheme=SCHEMES[scheme], with_bias=a.get("with_bias", 0), tied_output=int(tied_output),
                     seed=seed, w_std=w_std, n_threads=n_threads)
    if native()[1].dfc_synth_model(str(path).encode(), C.byref(spec)) != 0:
        raise DiffuseError(_dfc_err())
    return str(path)


def quantize_file(src, dst, qtype: str, n_threads: int = 0):
    if native()[1].dfc_quantize_file(str(src).encode(), str(dst).encode(), qtype.encode(), n_threads) != 0:
        raise DiffuseError(_dfc_err())


def tokens_to_unmask(step, total_steps, total_masked, schedule=COSINE) -> int:
    return native()[1].dfc_tokens_to_unmask(step, total_steps, total_masked, schedule)


@dataclass
class HParams:
    n_vocab: int
    n_embd: int
    n_head: int
    n_head_kv: int
    n_layer: int
    n_ff: int
    n_ctx_max: int
    mask_token_id: int
    is_dream: bool
    rope_theta: float
    rms_norm_eps: float


def tp_unique_id() -> bytes:
    """A fresh NCCL id for a tensor-parallel group (one rank creates it, every rank passes it)."""
    buf = np.zeros(128, np.uint8)
    if native()[0].dfb_tp_unique_id(_ptr(buf), buf.size) != 0:
        raise DiffuseError(_dfb_err())
    return buf.tobytes()


class Model:
    """diffuse_model: GGUF parsed and uploaded to the current CUDA device (DIFFUSE_DEVICE
    selects another).  tp=(rank, size, nccl_id): this rank's slice of a tensor-parallel group
    (every rank loads at the same time); logits then hold the rank's vocabulary columns
    [tp_v0, tp_v0 + tp_vocab)."""

    def __init__(self, path, n_threads: int = 4, tp=None):
        if tp is None:
            self._h = native()[1].dfc_model_load(str(path).encode(), n_threads)
        else:
            rank, size, nid = tp
            idb = np.frombuffer(bytes(nid), np.uint8).copy()
            self._h = native()[1].dfc_model_load_tp(str(path).encode(), rank, size, _ptr(idb), idb.size)
        if not self._h:
            raise DiffuseError(_dfc_err())
        i = np.zeros(9, np.int32)
        f = np.zeros(2, np.float32)
        native()[1].dfc_model_hparams(self._h, _ptr(i), _ptr(f))
        self.hparams = HParams(*[int(v) for v in i[:8]], bool(i[8]), float(f[0]), float(f[1]))
        t = np.zeros(4, np.int32)
        native()[1].dfc_model_tp_info(self._h, _ptr(t[0:]), _ptr(t[1:]), _ptr(t[2:]), _ptr(t[3:]))
        self.tp_rank, self.tp_size, self.tp_v0, self.tp_vocab = (int(v) for v in t)

    def close(self):
        if self._h:
            native()[1].dfc_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Context:
    """diffuse_context: device buffers + stream of one generation at a time."""

    def __init__(self, model: Model, n_ctx: int = 0, n_threads: int = 4):
        self.model = model
        self._h = native()[1].dfc_context_new(model._h, n_ctx, n_threads)
        if not self._h:
            raise DiffuseError(_dfc_err())
        self.engine = native()[1].dfc_context_engine(self._h)

    def forward(self, tokens) -> np.ndarray:
        """diffuse_forward: logits [n, n_vocab] for n tokens (no cache); a tensor-parallel
        rank gets its vocabulary columns [n, tp_vocab]."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.empty((t.size, self.model.tp_vocab), dtype=np.float32)
        if not native()[1].dfc_forward(self._h, _ptr(t), t.size, _ptr(out)):
            raise DiffuseError(_dfc_err())
        return out

    def linear(self, role: int, layer: int, x: np.ndarray) -> np.ndarray:
        """y = x . W^T through the production dequant GEMM (for parity tests)."""
        hp = self.model.hparams
        x = np.ascontiguousarray(x, dtype=np.float32)
        kv = hp.n_head_kv * (hp.n_embd // hp.n_head)
        n_out = {OUTPUT: hp.n_vocab, WQ: hp.n_embd, WK: kv, WV: kv, WO: hp.n_embd, GATE: hp.n_ff, UP: hp.n_ff,
                 DOWN: hp.n_embd}[role]
        y = np.empty((x.shape[0], n_out), dtype=np.float32)
        if native()[0].dfb_linear(self.engine, role, layer, _ptr(x), x.shape[0], _ptr(y)) != 0:
            raise DiffuseError(_dfb_err())
        return y

    def generate(self, prompt, n_generate: int, params: SamplerParams | None = None, trace: bool = False):
        """diffuse_generate: returns generated ids (and a per-step trace dict)."""
        params = params or SamplerParams()
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.empty(n_generate, dtype=np.int32)
        tr = None
        if trace:
            S = params.n_steps
            arrs = dict(n_active=np.zeros(S, np.int32), n_unmasked=np.zeros(S, np.int32),
                        commit_pos=np.full(S * n_generate, -1, np.int32), commit_tok=np.full(S * n_generate, -1, np.int32),
                        fwd_ms=np.zeros(S, np.float32), step_ms=np.zeros(S, np.float32))
            tr = Trace(max_steps=S, **{k: v.ctypes.data_as(C.POINTER(C.c_int32 if v.dtype == np.int32 else C.c_float))
                                       for k, v in arrs.items()})
        rc = native()[1].dfc_generate(self._h, _ptr(p), p.size, n_generate, C.byref(params), _ptr(out),
                                      C.byref(tr) if tr is not None else None)
        if rc < 0:
            raise DiffuseError(_dfc_err())
        if not trace:
            return out
        info = {k: v for k, v in arrs.items()}
        info["steps_run"] = tr.steps_run
        info["total_ms"] = tr.total_ms
        info["commit_pos"] = info["commit_pos"].reshape(params.n_steps, n_generate)
        info["commit_tok"] = info["commit_tok"].reshape(params.n_steps, n_generate)
        return out, info

    def generate_batch(self, prompts, n_generate: int, params: SamplerParams | None = None, trace: bool = False):
        """Several independent sequences (prompts: list of 1-D id arrays, any lengths),
        each running diffuse_generate's loop as alone, stepped together in one forward per
        step.  Returns ids [n_seq, n_generate] (and a per-step trace dict)."""
        params = params or SamplerParams()
        ps = [np.ascontiguousarray(p, dtype=np.int32) for p in prompts]
        lens = np.array([p.size for p in ps], np.int32)
        cat = np.ascontiguousarray(np.concatenate(ps) if lens.sum() else np.zeros(1, np.int32), dtype=np.int32)
        n = len(ps)
        out = np.empty((n, n_generate), dtype=np.int32)
        tr = None
        if trace:
            S = params.n_steps
            arrs = dict(n_active=np.zeros((S, n), np.int32), n_unmasked=np.zeros((S, n), np.int32),
                        fwd_ms=np.zeros(S, np.float32), step_ms=np.zeros(S, np.float32))
            tr = BatchTrace(max_steps=S, **{k: v.ctypes.data_as(C.POINTER(C.c_int32 if v.dtype == np.int32 else C.c_float))
                                            for k, v in arrs.items()})
        rc = native()[1].dfc_generate_batch(self._h, _ptr(cat), _ptr(lens), n, n_generate, C.byref(params), _ptr(out),
                                            C.byref(tr) if tr is not None else None)
        if rc < 0:
            raise DiffuseError(_dfc_err())
        if not trace:
            return out
        info = dict(arrs)
        info["steps_run"] = tr.steps_run
        info["total_ms"] = tr.total_ms
        return out, info

    # ── step-level access to the device loop (teacher-forced parity checks) ──
    def gen_begin(self, prompt, n_generate: int, params: SamplerParams):
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        if native()[0].dfb_gen_begin(self.engine, _ptr(p), p.size, n_generate, C.byref(params)) != 0:
            raise DiffuseError(_dfb_err())
        self._total = p.size + n_generate

    def gen_set_uniforms(self, u):
        """temperature > 0: the next step's uniforms (one per masked position, position order)."""
        a = np.ascontiguousarray(u, dtype=np.float64)
        if native()[0].dfb_gen_set_uniforms(self.engine, _ptr(a) if a.size else None, a.size) != 0:
            raise DiffuseError(_dfb_err())

    def gen_step(self, step: int, n_unmask: int, force_full: bool, order=None) -> dict:
        st = np.zeros(6, np.int32)  # dfb_step_stats: 4 ints + 2 floats
        o = None if order is None else np.ascontiguousarray(order, dtype=np.int32)
        rc = native()[0].dfb_gen_step(self.engine, step, n_unmask, int(force_full), None if o is None else _ptr(o), _ptr(st))
        if rc != 0:
            raise DiffuseError(_dfb_err())
        f = st[4:].view(np.float32)
        return dict(n_active=int(st[0]), n_unmasked=int(st[1]), n_masked=int(st[2]), used_cache=int(st[3]),
                    fwd_ms=float(f[0]), step_ms=float(f[1]))

    def gen_begin_batch(self, prompts, n_generate: int, params: SamplerParams):
        ps = [np.ascontiguousarray(p, dtype=np.int32) for p in prompts]
        lens = np.array([p.size for p in ps], np.int32)
        gens = np.full(len(ps), n_generate, np.int32)
        cat = np.ascontiguousarray(np.concatenate(ps) if lens.sum() else np.zeros(1, np.int32), dtype=np.int32)
        if native()[0].dfb_gen_begin_batch(self.engine, len(ps), _ptr(cat), _ptr(lens), _ptr(gens), C.byref(params)) != 0:
            raise DiffuseError(_dfb_err())
        self._total = int(lens.sum()) + n_generate * len(ps)
        self._n_seq = len(ps)

    def gen_step_batch(self, step: int, n_unmask, force_full: bool, orders=None) -> list:
        sched = np.ascontiguousarray(n_unmask, dtype=np.int32)
        st = np.zeros((self._n_seq, 6), np.int32)
        o = None if orders is None else np.ascontiguousarray(orders, dtype=np.int32)
        rc = native()[0].dfb_gen_step_batch(self.engine, step, _ptr(sched), int(force_full),
                                            None if o is None else _ptr(o), _ptr(st))
        if rc != 0:
            raise DiffuseError(_dfb_err())
        f = st[:, 4:].copy().view(np.float32)
        return [dict(n_active=int(r[0]), n_unmasked=int(r[1]), n_masked=int(r[2]), used_cache=int(r[3]),
                     fwd_ms=float(f[i, 0]), step_ms=float(f[i, 1])) for i, r in enumerate(st)]

    def gen_commits_batch(self):
        pos = np.empty(self._total, np.int32)
        tok = np.empty(self._total, np.int32)
        cnt = np.zeros(self._n_seq, np.int32)
        n = native()[0].dfb_gen_commits_batch(self.engine, _ptr(pos), _ptr(tok), _ptr(cnt), self._total)
        if n < 0:
            raise DiffuseError(_dfb_err())
        out, w = [], 0
        for c in cnt.tolist():
            out.append((pos[w:w + c].copy(), tok[w:w + c].copy()))
            w += c
        return out

    def gen_tokens(self) -> np.ndarray:
        out = np.empty(self._total, np.int32)
        if native()[0].dfb_gen_tokens(self.engine, _ptr(out), out.size) != 0:
            raise DiffuseError(_dfb_err())
        return out

    def gen_commits(self):
        pos = np.empty(self._total, np.int32)
        tok = np.empty(self._total, np.int32)
        n = native()[0].dfb_gen_commits(self.engine, _ptr(pos), _ptr(tok), self._total)
        if n < 0:
            raise DiffuseError(_dfb_err())
        return pos[:n], tok[:n]

    # ── direct access to the device state of the current generation ──
    def logits_rows(self, row0: int, nrows: int) -> np.ndarray:
        out = np.empty((nrows, self.model.tp_vocab), dtype=np.float32)
        if native()[0].dfb_gen_logits(self.engine, row0, nrows, _ptr(out)) != 0:
            raise DiffuseError(_dfb_err())
        return out

    def close(self):
        if self._h:
            native()[1].dfc_context_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


from . import dp  # noqa: E402  (data-parallel plumbing over independent sequences)
from . import serve  # noqa: E402  (request server over a pool of contexts)
from . import tp  # noqa: E402  (tensor-parallel shard plan and its numpy execution)
