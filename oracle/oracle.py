"""ctypes binding of the CPU oracle (liboracle.so) — TEST INFRASTRUCTURE ONLY.

Imported by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
--impl reference legs, as the checker.  The product never loads it.
"""
from __future__ import annotations

import ctypes as C
import pathlib
import subprocess

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
EXACT, GGML = 0, 1


class SamplerParams(C.Structure):
    _fields_ = [("n_steps", C.c_int32), ("temperature", C.c_float), ("schedule", C.c_int32),
                ("remasking", C.c_int32), ("seed", C.c_uint32), ("entropy_threshold", C.c_float),
                ("use_cache", C.c_int32), ("cache_refresh", C.c_int32), ("cache_keep_active", C.c_int32)]

    def __init__(self, **kw):
        d = dict(n_steps=32, temperature=0.0, schedule=0, remasking=0, seed=42, entropy_threshold=1.5,
                 use_cache=1, cache_refresh=0, cache_keep_active=0)
        d.update(kw)
        super().__init__(**{k: (int(v) if isinstance(v, bool) else v) for k, v in d.items()})


class SynthSpec(C.Structure):
    _fields_ = [("is_dream", C.c_int32), ("n_vocab", C.c_int32), ("n_embd", C.c_int32), ("n_head", C.c_int32),
                ("n_head_kv", C.c_int32), ("n_layer", C.c_int32), ("n_ff", C.c_int32), ("n_ctx", C.c_int32),
                ("mask_token_id", C.c_int32), ("rope_theta", C.c_float), ("rms_norm_eps", C.c_float),
                ("scheme", C.c_int32), ("with_bias", C.c_int32), ("tied_output", C.c_int32),
                ("seed", C.c_uint64), ("w_std", C.c_float), ("n_threads", C.c_int32)]


SCHEMES = {"f32": 0, "f16": 1, "q8_0": 2, "q4_k_m": 3}


def synth_model(path, arch: dict, scheme: str = "q4_k_m", seed: int = 0, w_std: float = 0.02,
                tied_output: bool = False, n_threads: int = 0, **overrides):
    """Seeded random-init GGUF written by the oracle alone (no product library): the
    same bytes as the product's synthesizer for the same arguments."""
    a = dict(arch)
    a.update(overrides)
    spec = SynthSpec(is_dream=a["is_dream"], n_vocab=a["n_vocab"], n_embd=a["n_embd"], n_head=a["n_head"],
                     n_head_kv=a["n_head_kv"], n_layer=a["n_layer"], n_ff=a["n_ff"], n_ctx=a.get("n_ctx", 4096),
                     mask_token_id=a["mask_token_id"], rope_theta=a["rope_theta"], rms_norm_eps=a["rms_norm_eps"],
                     scheme=SCHEMES[scheme], with_bias=a.get("with_bias", 0), tied_output=int(tied_output),
                     seed=seed, w_std=w_std, n_threads=n_threads)
    if lib().orc_synth_model(str(path).encode(), C.byref(spec)) != 0:
        raise ValueError(f"oracle synth failed for {path}")
    return str(path)


class _Trace(C.Structure):
    _fields_ = [("max_steps", C.c_int32), ("n_gen", C.c_int32), ("steps_run", C.c_int32),
                ("n_active", C.POINTER(C.c_int32)), ("n_unmask", C.POINTER(C.c_int32)),
                ("commit_pos", C.POINTER(C.c_int32)), ("commit_tok", C.POINTER(C.c_int32)),
                ("final_logits", C.POINTER(C.c_float))]


_lib = None


def lib():
    global _lib
    if _lib is None:
        so = HERE / "liboracle.so"
        if not so.exists():
            subprocess.run(["make", "-C", str(HERE)], check=True, capture_output=True)
        _lib = C.CDLL(str(so))
        P, I = C.c_void_p, C.c_int32
        for name, res, args in [
            ("orc_load", P, [C.c_char_p]), ("orc_free", None, [P]), ("orc_hparams", I, [P, P, P]),
            ("orc_tensor", I, [P, C.c_char_p, P, P, P, P]), ("orc_dequantize", I, [I, P, C.c_int64, P]),
            ("orc_matmul", I, [P, C.c_char_p, P, I, P, I, I]), ("orc_forward", I, [P, P, I, P, I, I]),
            ("orc_forward_layers", I, [P, P, I, P, I, I, I]),
            ("orc_generate", I, [P, P, I, I, C.POINTER(SamplerParams), P, C.POINTER(_Trace), I, I]),
            ("orc_sampler_step", I, [P, I, I, P, P, I, I, C.POINTER(SamplerParams), P, P, P, P]),
            ("orc_tokens_to_unmask", I, [I, I, I, I]), ("orc_entropy", C.c_float, [P, I]),
            ("orc_rope_table", I, [I, I, C.c_float, P, P]),
            ("orc_sess_new", P, [P, P, I, I, C.POINTER(SamplerParams), I, I]), ("orc_sess_free", None, [P]),
            ("orc_sess_forward", I, [P, I]), ("orc_sess_sample", I, [P, I, P, P]), ("orc_sess_commit", I, [P, P, P, I]),
            ("orc_sess_logits", I, [P, I, I, P]), ("orc_sess_tokens", I, [P, P]),
            ("orc_synth_model", I, [C.c_char_p, C.POINTER(SynthSpec)]),
            ("orc_sample_row", I, [P, I, C.c_float, C.c_double, P, P]),
            ("orc_canonical", I, [C.c_uint32, I, P]),
        ]:
            fn = getattr(_lib, name)
            fn.restype, fn.argtypes = res, args
    return _lib


def _p(a):
    return a.ctypes.data_as(C.c_void_p)


def dequantize(raw: np.ndarray, ggml_type: int, n: int) -> np.ndarray:
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    out = np.empty(n, np.float32)
    if lib().orc_dequantize(ggml_type, _p(raw), n, _p(out)) != 0:
        raise ValueError("bad dequantize arguments")
    return out


def tokens_to_unmask(step, total, masked, schedule=0):
    return lib().orc_tokens_to_unmask(step, total, masked, schedule)


def entropy(row: np.ndarray) -> float:
    row = np.ascontiguousarray(row, dtype=np.float32)
    return float(lib().orc_entropy(_p(row), row.size))


def rope_table(n_pos, n_dims, base):
    c = np.empty((n_pos, n_dims // 2), np.float32)
    s = np.empty_like(c)
    lib().orc_rope_table(n_pos, n_dims, base, _p(c), _p(s))
    return c, s


def sampler_step(logits_full, seq, is_masked, is_dream, step, params: SamplerParams):
    """One reference sampler decision on given logits (updates seq / is_masked copies)."""
    logits_full = np.ascontiguousarray(logits_full, dtype=np.float32)
    seq = np.array(seq, dtype=np.int32)
    msk = np.array(is_masked, dtype=np.uint8)
    n = int(msk.sum())
    cp = np.full(max(n, 1), -1, np.int32)
    ct = np.full(max(n, 1), -1, np.int32)
    ent = np.zeros(max(n, 1), np.float32)
    conf = np.zeros(max(n, 1), np.float32)
    k = lib().orc_sampler_step(_p(logits_full), logits_full.shape[1], seq.size, _p(seq), _p(msk), int(is_dream),
                               step, C.byref(params), _p(cp), _p(ct), _p(ent), _p(conf))
    return dict(n=k, pos=cp[:k], tok=ct[:k], entropy=ent[:n], conf=conf[:n], seq=seq, masked=msk)


def sample_row(row, temperature: float, u: float):
    """The reference's temperature > 0 draw on one logits row with the uniform given:
    (token, its probability, distance from u to the nearest bounding cumulative sum)."""
    row = np.ascontiguousarray(row, dtype=np.float32)
    conf = np.zeros(1, np.float32)
    margin = np.zeros(1, np.float64)
    k = lib().orc_sample_row(_p(row), row.size, float(temperature), float(u), _p(conf), _p(margin))
    return int(k), float(conf[0]), float(margin[0])


def canonical(seed: int, n: int) -> np.ndarray:
    """The uniforms std::discrete_distribution draws from std::mt19937(seed)."""
    out = np.zeros(max(n, 1), np.float64)
    lib().orc_canonical(seed, n, _p(out))
    return out[:n]


class OracleModel:
    def __init__(self, path):
        self.h = lib().orc_load(str(path).encode())
        if not self.h:
            raise ValueError(f"oracle cannot load {path}")
        i = np.zeros(9, np.int32)
        f = np.zeros(2, np.float32)
        lib().orc_hparams(self.h, _p(i), _p(f))
        (self.n_vocab, self.n_embd, self.n_head, self.n_head_kv, self.n_layer, self.n_ff, self.n_ctx_max,
         self.mask_token_id, is_dream) = [int(v) for v in i]
        self.is_dream = bool(is_dream)
        self.rope_theta, self.eps = float(f[0]), float(f[1])

    def tensor(self, name):
        t, n0, n1, d = C.c_int32(), C.c_int64(), C.c_int64(), C.c_void_p()
        if lib().orc_tensor(self.h, name.encode(), C.byref(t), C.byref(n0), C.byref(n1), C.byref(d)) != 0:
            raise KeyError(name)
        return t.value, n0.value, n1.value, d.value

    def matmul(self, name, x, mode=EXACT, n_threads=0):
        x = np.ascontiguousarray(x, dtype=np.float32)
        _, k, n, _ = self.tensor(name)
        y = np.empty((x.shape[0], n), np.float32)
        if lib().orc_matmul(self.h, name.encode(), _p(x), x.shape[0], _p(y), mode, n_threads) != 0:
            raise KeyError(name)
        return y

    def forward(self, tokens, mode=EXACT, n_threads=0):
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.empty((t.size, self.n_vocab), np.float32)
        lib().orc_forward(self.h, _p(t), t.size, _p(out), mode, n_threads)
        return out

    def forward_layers(self, tokens, n_layers, mode=EXACT, n_threads=0):
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.empty((t.size, self.n_vocab), np.float32)
        lib().orc_forward_layers(self.h, _p(t), t.size, _p(out), mode, n_threads, n_layers)
        return out

    def generate(self, prompt, n_gen, params: SamplerParams, mode=EXACT, n_threads=0, final_logits=False):
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.empty(n_gen, np.int32)
        S = params.n_steps
        arr = dict(n_active=np.zeros(S, np.int32), n_unmask=np.zeros(S, np.int32),
                   commit_pos=np.full(S * n_gen, -1, np.int32), commit_tok=np.full(S * n_gen, -1, np.int32))
        fl = np.empty((p.size + n_gen, self.n_vocab), np.float32) if final_logits else None
        tr = _Trace(max_steps=S, n_gen=n_gen, steps_run=0,
                    **{k: v.ctypes.data_as(C.POINTER(C.c_int32)) for k, v in arr.items()},
                    final_logits=fl.ctypes.data_as(C.POINTER(C.c_float)) if fl is not None else None)
        lib().orc_generate(self.h, _p(p), p.size, n_gen, C.byref(params), _p(out), C.byref(tr), mode, n_threads)
        arr["steps_run"] = tr.steps_run
        arr["commit_pos"] = arr["commit_pos"].reshape(S, n_gen)
        arr["commit_tok"] = arr["commit_tok"].reshape(S, n_gen)
        if fl is not None:
            arr["final_logits"] = fl
        return out, arr

    def close(self):
        if self.h:
            lib().orc_free(self.h)
            self.h = None


class OracleSession:
    """One diffuse_sample run of the oracle, step by step (teacher-forced checks): the
    forward of a step by the reference's full / cached rules, the session's own sampler
    decision, or commits decided elsewhere."""

    def __init__(self, model: OracleModel, prompt, n_gen, params: SamplerParams, mode=EXACT, n_threads=0):
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        self.model, self.n_prompt, self.n_gen, self.total = model, p.size, n_gen, p.size + n_gen
        self.params = params
        self.h = lib().orc_sess_new(model.h, _p(p), p.size, n_gen, C.byref(params), mode, n_threads)

    def forward(self, step: int) -> int:
        return lib().orc_sess_forward(self.h, step)

    def sample(self, step: int):
        cp = np.full(max(self.n_gen, 1), -1, np.int32)
        ct = np.full(max(self.n_gen, 1), -1, np.int32)
        k = lib().orc_sess_sample(self.h, step, _p(cp), _p(ct))
        return cp[:k], ct[:k]

    def commit(self, pos, tok):
        pos = np.ascontiguousarray(pos, dtype=np.int32)
        tok = np.ascontiguousarray(tok, dtype=np.int32)
        if lib().orc_sess_commit(self.h, _p(pos), _p(tok), pos.size) != 0:
            raise ValueError("commit at a position that is not masked")

    def logits(self, row0=0, nrows=None):
        nrows = self.total - row0 if nrows is None else nrows
        out = np.empty((nrows, self.model.n_vocab), np.float32)
        if lib().orc_sess_logits(self.h, row0, nrows, _p(out)) != 0:
            raise ValueError("rows out of range")
        return out

    def tokens(self):
        out = np.empty(self.total, np.int32)
        n_masked = lib().orc_sess_tokens(self.h, _p(out))
        return out, n_masked

    def close(self):
        if self.h:
            lib().orc_sess_free(self.h)
            self.h = None

    def __del__(self):
        self.close()
