"""dfb_linear_noalloc: the allocation-free linear layer, for callers that cannot
allocate device memory while they run (a serving stack whose caching allocator owns
all device memory, or code that cannot take the device-wide synchronization that
cudaMalloc / cudaFree can cause).  Its GEMM scratch is a fixed array inside the
library; the test owns every buffer it passes in.

The model is built straight through the C-ABI (dfb_model_create / set_tensor /
finalize) and each result is checked, on two calls in a row, against an f64 product of
the dequantized weight and against the existing entry point dfb_linear on the same
weight and input.  The two entry points split their operands differently (plain f16
activations with f32-dequantized hi / lo weights here; pair-row activations and the f16
dequant routes in dfb_linear), so they agree to the GEMM's accuracy against the exact
product (3e-5 mean relative), not bit for bit.  This file sorts last so that a run
stopping at the first failure has run every other test already.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import MINI_LLADA, metrics

pytestmark = pytest.mark.gpu

ROLES = {"token_embd.weight": (0, 0), "output_norm.weight": (1, 0), "output.weight": (2, 0)}
LAYER_ROLES = {"attn_norm.weight": 3, "attn_q.weight": 4, "attn_k.weight": 5, "attn_v.weight": 6,
               "attn_output.weight": 7, "ffn_norm.weight": 11, "ffn_gate.weight": 12, "ffn_up.weight": 13,
               "ffn_down.weight": 14}


class HParams(C.Structure):
    _fields_ = [("n_vocab", C.c_int32), ("n_embd", C.c_int32), ("n_head", C.c_int32), ("n_head_kv", C.c_int32),
                ("n_layer", C.c_int32), ("n_ff", C.c_int32), ("n_ctx_max", C.c_int32), ("mask_token_id", C.c_int32),
                ("rope_theta", C.c_float), ("rms_norm_eps", C.c_float), ("shift_logits", C.c_int32)]


@pytest.fixture(scope="module")
def engine_model(pkg, tmp_path_factory):
    import gguf
    path = pkg.synth_model(tmp_path_factory.mktemp("noalloc") / "m.gguf", MINI_LLADA, "q4_k_m", seed=21, n_layer=3)
    dfb, _ = pkg.native()
    dfb.dfb_model_create.argtypes = [C.POINTER(HParams), C.c_int, C.POINTER(C.c_void_p)]
    dfb.dfb_model_set_tensor.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int64, C.c_int64, C.c_void_p,
                                         C.c_size_t]
    dfb.dfb_model_finalize.argtypes = [C.c_void_p]
    dfb.dfb_model_free.argtypes = [C.c_void_p]
    dfb.dfb_ctx_create.argtypes = [C.c_void_p, C.c_int, C.POINTER(C.c_void_p)]
    dfb.dfb_ctx_free.argtypes = [C.c_void_p]
    dfb.dfb_linear_noalloc.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]
    a = MINI_LLADA
    hp = HParams(a["n_vocab"], a["n_embd"], a["n_head"], a["n_head_kv"], 3, a["n_ff"], 4096, a["mask_token_id"],
                 a["rope_theta"], a["rms_norm_eps"], 0)
    m = C.c_void_p()
    assert dfb.dfb_model_create(C.byref(hp), -1, C.byref(m)) == 0, dfb.dfb_last_error()
    reader = gguf.GGUFReader(path)
    weights = {}
    keep = []
    for t in reader.tensors:
        if t.name in ROLES:
            role, layer = ROLES[t.name]
        else:
            _, li, rest = t.name.split(".", 2)
            role, layer = LAYER_ROLES[rest], int(li)
        data = np.ascontiguousarray(t.data)
        keep.append(data)
        ne1 = int(t.shape[1]) if len(t.shape) > 1 else 1
        weights[(role, layer)] = t
        rc = dfb.dfb_model_set_tensor(m, role, layer, int(t.tensor_type), int(t.shape[0]), ne1,
                                      data.ctypes.data_as(C.c_void_p), int(t.n_bytes))
        assert rc == 0, dfb.dfb_last_error()
    assert dfb.dfb_model_finalize(m) == 0, dfb.dfb_last_error()
    ctx = C.c_void_p()
    assert dfb.dfb_ctx_create(m, 0, C.byref(ctx)) == 0, dfb.dfb_last_error()
    yield dfb, m, ctx, weights
    dfb.dfb_ctx_free(ctx)
    dfb.dfb_model_free(m)


@pytest.mark.parametrize("role,layer,k,n_out", [(7, 1, 1024, 1024), (14, 0, 2816, 1024), (14, 1, 2816, 1024),
                                                (2, 0, 1024, 5000)],
                         ids=["attn_output-q4k", "ffn_down-q6k", "ffn_down-q4k", "output-q6k"])
@pytest.mark.parametrize("M", [17, 256])
def test_noalloc_matches_dfb_linear(engine_model, role, layer, k, n_out, M):
    import gguf
    import torch
    dfb, m, ctx, weights = engine_model
    x16 = (np.random.default_rng(M + role).standard_normal((M, k)) * 0.5).astype(np.float16)
    ref = np.empty((M, n_out), np.float32)
    x32 = np.ascontiguousarray(x16.astype(np.float32))
    assert dfb.dfb_linear(ctx, role, layer, x32.ctypes.data_as(C.c_void_p), M,
                          ref.ctypes.data_as(C.c_void_p)) == 0, dfb.dfb_last_error()
    t = weights[(role, layer)]
    w = gguf.quants.dequantize(t.data, t.tensor_type).reshape(n_out, k).astype(np.float64)
    exact = x32.astype(np.float64) @ w.T
    mx, rel = metrics(ref, exact)
    assert rel < 3e-5, (mx, rel)
    xd = torch.from_numpy(x16).cuda()
    for it in range(2):  # the scratch keeps the previous call's contents
        yd = torch.full((M, n_out), float("nan"), dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        rc = dfb.dfb_linear_noalloc(m, role, layer, C.c_void_p(xd.data_ptr()), M, C.c_void_p(yd.data_ptr()), None)
        assert rc == 0, dfb.dfb_last_error()
        torch.cuda.synchronize()
        if it:  # after the first call on the device nothing is allocated
            assert torch.cuda.mem_get_info()[0] >= free0
        got = yd.cpu().numpy()
        assert np.isfinite(got).all()
        mx, rel = metrics(got, exact)
        assert rel < 3e-5, (mx, rel)
        mx, rel = metrics(got, ref)
        assert rel < 5e-5 and mx < 1e-3 * max(1.0, float(np.abs(ref).max())), (mx, rel)


def test_noalloc_rejects_oversize_and_fused(engine_model):
    import torch
    dfb, m, ctx, _ = engine_model
    xd = torch.zeros((300, 1024), dtype=torch.float16, device="cuda")
    yd = torch.zeros((300, 1024), dtype=torch.float32, device="cuda")
    assert dfb.dfb_linear_noalloc(m, 7, 0, C.c_void_p(xd.data_ptr()), 300, C.c_void_p(yd.data_ptr()), None) == -1
    assert b"outside" in dfb.dfb_last_error()
    assert dfb.dfb_linear_noalloc(m, 4, 0, C.c_void_p(xd.data_ptr()), 8, C.c_void_p(yd.data_ptr()), None) == -6
