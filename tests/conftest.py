"""Shared fixtures: the product package (loaded by path: its directory name has a
hyphen), the CPU oracle binding, and GGUF fixtures."""
import importlib.util
import json
import pathlib
import sys

import numpy as np
import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def load_package():
    name = "diffuse_b200"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, ROOT / "diffuse-cpp_b200" / "__init__.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def pkg():
    return load_package()


@pytest.fixture(scope="session")
def orc():
    from oracle import oracle
    return oracle


# The tiny LLaDA-shaped model of the reference's tests/test-e2e.py:17-71 (hidden 64,
# 4 heads, 2 layers, vocab 256, ff 128, mask 200, N(0,1) weights from
# default_rng(42), norms 1), written with gguf-py the way tools/convert-llada.py
# writes it (arch "diffuse", same metadata keys and tensor names).
TINY = dict(hidden=64, heads=4, layers=2, vocab=256, ff=128, mask=200)


def write_tiny_gguf(path, dtype=np.float32, dream=False, kv_heads=None, seed=42, bias=False, drop=(), as_q5_0=(),
                    wrong_shape=()):
    """drop: tensor names left out; as_q5_0: tensors written with GGML type Q5_0 (a type
    the engine does not take); wrong_shape: tensors written with one row too many."""
    import gguf
    t = TINY
    kvh = kv_heads or t["heads"]
    hd = t["hidden"] // t["heads"]
    rng = np.random.default_rng(seed)
    w = gguf.GGUFWriter(str(path), arch="diffuse")
    w.add_name("tiny")
    w.add_block_count(t["layers"])
    w.add_head_count(t["heads"])
    w.add_head_count_kv(kvh)
    w.add_embedding_length(t["hidden"])
    w.add_feed_forward_length(t["ff"])
    w.add_context_length(512)
    w.add_vocab_size(t["vocab"])
    w.add_rope_freq_base(500000.0)
    w.add_layer_norm_rms_eps(1e-5)
    w.add_uint32("diffuse.mask_token_id", t["mask"])
    w.add_string("diffuse.model_type", "dream" if dream else "llada")
    H, V, F = t["hidden"], t["vocab"], t["ff"]
    def mat(r, c):
        return rng.standard_normal((r, c)).astype(np.float32).astype(dtype)
    add = w.add_tensor

    def add_tensor(name, arr):
        if name in drop:
            return
        if name in wrong_shape:
            arr = np.concatenate([arr, arr[:1]], axis=0)
        if name in as_q5_0:  # 22 bytes per block of 32 values
            rows = arr.shape[0] if arr.ndim > 1 else 1
            n = arr.shape[-1]
            add(name, np.zeros((rows, n // 32 * 22), np.uint8), raw_dtype=gguf.GGMLQuantizationType.Q5_0)
            return
        add(name, arr)
    w.add_tensor = add_tensor
    w.add_tensor("token_embd.weight", mat(V, H))
    w.add_tensor("output_norm.weight", np.ones(H, np.float32).astype(dtype))
    w.add_tensor("output.weight", mat(V, H))
    for i in range(t["layers"]):
        p = f"blk.{i}."
        w.add_tensor(p + "attn_norm.weight", np.ones(H, np.float32).astype(dtype))
        w.add_tensor(p + "attn_q.weight", mat(H, H))
        w.add_tensor(p + "attn_k.weight", mat(kvh * hd, H))
        w.add_tensor(p + "attn_v.weight", mat(kvh * hd, H))
        if bias:
            w.add_tensor(p + "attn_q.bias", rng.standard_normal(H).astype(np.float32))
            w.add_tensor(p + "attn_k.bias", rng.standard_normal(kvh * hd).astype(np.float32))
            w.add_tensor(p + "attn_v.bias", rng.standard_normal(kvh * hd).astype(np.float32))
        w.add_tensor(p + "attn_output.weight", mat(H, H))
        w.add_tensor(p + "ffn_norm.weight", np.ones(H, np.float32).astype(dtype))
        w.add_tensor(p + "ffn_gate.weight", mat(F, H))
        w.add_tensor(p + "ffn_up.weight", mat(F, H))
        w.add_tensor(p + "ffn_down.weight", mat(H, F))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return str(path)


# Reduced-depth / reduced-width models with the real head geometry (head_dim 128,
# MHA for LLaDA, GQA 7:1 for Dream), K dims multiples of 256 for the K-quants.
MINI_LLADA = dict(is_dream=0, n_vocab=5000, n_embd=1024, n_head=8, n_head_kv=8, n_layer=2, n_ff=2816,
                  n_ctx=4096, mask_token_id=4999, rope_theta=500000.0, rms_norm_eps=1e-5, with_bias=0)
MINI_DREAM = dict(is_dream=1, n_vocab=6000, n_embd=1792, n_head=14, n_head_kv=2, n_layer=2, n_ff=4864,
                  n_ctx=4096, mask_token_id=5999, rope_theta=1000000.0, rms_norm_eps=1e-6, with_bias=1)


@pytest.fixture(scope="session")
def model_dir(tmp_path_factory):
    return tmp_path_factory.mktemp("models")


def metrics(a, b):
    """max-abs and mean relative error sum|a-b| / sum|b| (the north-star logits metrics)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    d = np.abs(a - b)
    return float(d.max()), float(d.sum() / max(np.abs(b).sum(), 1e-30))
