"""Logits of the full-depth headline architectures against the CPU oracle (needs a B200).

LLaDA-8B (32 layers, Q4_K_M) on the step-0 sequence of config 1 (16 prompt ids + 64
mask ids) and Dream-7B (28 layers, GQA 28/4, q/k/v bias, Q4_K_M) on the step-0 sequence
of config 3 (128 prompt ids + 64 mask ids), both through dfb_forward (diffuse_forward,
diffuse-graph.cpp:676-680), held to the north-star bounds against the oracle's exact mode.

The oracle's GGML-emulation mode (Q8_K / Q8_0 activation quantization before every
weight matmul, as GGML's CPU mul_mat does) is reported beside it, not asserted: that
arithmetic is chaotic at depth -- a one-ulp change of one layer-0 norm weight moves its
32-layer logits by ~1.5e-1 mean relative error (tests/test_host_cpu.py pins the effect on
a small model) -- so no implementation that is not bit-identical to GGML's float order
can be held to 1e-3 against it, while the exact mode moves by ~1e-5 under the same change.

The models are the bench's (same synthesis, same cache directory), so a bench run after
the tests reuses them.
"""
import os
import pathlib
import tempfile
import time

import numpy as np
import pytest

from conftest import metrics

pytestmark = pytest.mark.gpu

LOGIT_MAXABS, LOGIT_MEANREL = 2e-2, 1e-3


def _model(pkg, arch_name):
    work = pathlib.Path(os.environ.get("DFB_BENCH_DIR", tempfile.gettempdir())) / "dfb_bench"
    work.mkdir(parents=True, exist_ok=True)
    path = work / f"{arch_name}_q4_k_m_seed0.gguf"
    if not path.exists():
        tmp = path.with_suffix(".tmp")
        pkg.synth_model(tmp, pkg.LLADA_8B if arch_name == "llada" else pkg.DREAM_7B, "q4_k_m", seed=0)
        tmp.rename(path)
    return str(path)


@pytest.mark.parametrize("arch,n_prompt,n_block", [("llada", 16, 64), ("dream", 128, 64)],
                         ids=["llada8b-config1-step0", "dream7b-config3-step0"])
def test_full_depth_logits(pkg, orc, arch, n_prompt, n_block):
    path = _model(pkg, arch)
    model = pkg.Model(path)
    hp = model.hparams
    prompt = np.random.default_rng(1234).integers(0, hp.mask_token_id - 1, n_prompt).astype(np.int32)
    toks = np.concatenate([prompt, np.full(n_block, hp.mask_token_id, np.int32)])
    ctx = pkg.Context(model, toks.size)
    got = ctx.forward(toks)
    ctx.close()
    model.close()
    om = orc.OracleModel(path)
    t0 = time.perf_counter()
    ref = om.forward(toks, mode=orc.EXACT)
    t_exact = time.perf_counter() - t0
    ggml = om.forward(toks, mode=orc.GGML)
    om.close()
    mx, rel = metrics(got, ref)
    gmx, grel = metrics(got, ggml)
    emx, erel = metrics(ref, ggml)
    print(f"{arch} {hp.n_layer} layers, {toks.size} rows: GPU vs exact max-abs {mx:.3e} mean-rel {rel:.3e}; "
          f"GPU vs GGML-emulation max-abs {gmx:.3e} mean-rel {grel:.3e}; exact vs GGML-emulation max-abs "
          f"{emx:.3e} mean-rel {erel:.3e} (oracle exact forward {t_exact:.1f} s)")
    assert rel < LOGIT_MEANREL and mx < LOGIT_MAXABS, (mx, rel)
    # argmax differs only between near-tied logits of the reference
    pick = ref[np.arange(toks.size), got.argmax(-1)]
    assert (ref.max(-1) - pick <= 2 * mx + 1e-6).all()
