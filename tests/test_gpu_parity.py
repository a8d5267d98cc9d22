"""CUDA path against the CPU oracle (needs a B200).  Every call goes through the
C-ABI (libdfb_cuda.so / libdiffuse.so)."""
import ctypes as C

import numpy as np
import pytest

from conftest import MINI_DREAM, MINI_LLADA, metrics, write_tiny_gguf

pytestmark = pytest.mark.gpu

# north-star logits tolerances (max-abs, mean relative error sum|a-b|/sum|b|), against the
# oracle's exact mode (f32 mathematics on the dequantized weights)
LOGIT_MAXABS, LOGIT_MEANREL = 2e-2, 1e-3
# One linear layer against the exact (f64) product: the operand splits leave ~2^-17 per
# element; the measured error, 0.6-2.3e-5 for every weight type (F16 weights included), is
# the tensor core's f32 accumulation over K/16 steps, 20-30x the oracle's sequential f32
# sums; full-depth logits stay at ~1e-4 of the 1e-3 bound.
GEMM_MEANREL = 3e-5


@pytest.fixture(scope="module")
def models(pkg, model_dir):
    m = {}
    m["q4km"] = pkg.synth_model(model_dir / "llada_q4km.gguf", MINI_LLADA, "q4_k_m", seed=11, n_layer=3)
    m["q8_0"] = pkg.synth_model(model_dir / "llada_q80.gguf", MINI_LLADA, "q8_0", seed=12)
    m["f16"] = pkg.synth_model(model_dir / "llada_f16.gguf", MINI_LLADA, "f16", seed=13)
    m["dream"] = pkg.synth_model(model_dir / "dream_q4km.gguf", MINI_DREAM, "q4_k_m", seed=14)
    m["tiny"] = write_tiny_gguf(model_dir / "tiny.gguf")
    m["tiny_gqa"] = write_tiny_gguf(model_dir / "tiny_gqa.gguf", kv_heads=2, bias=True, dream=True)
    m["tied"] = pkg.synth_model(model_dir / "llada_tied.gguf", MINI_LLADA, "q4_k_m", seed=15, n_layer=2,
                                tied_output=True)
    # LLaDA-8B width, one layer: ~10 k-blocks per CTA pair per launch, as in the real model
    m["wide"] = pkg.synth_model(model_dir / "llada_wide.gguf", pkg.LLADA_8B, "q4_k_m", seed=16, n_layer=1,
                                n_vocab=16384)
    return m


GEMM_CASES = [  # (model, role, layer, tensor name, expected GGML type)
    ("q4km", "WQ", 1, "blk.1.attn_q.weight", 12), ("q4km", "WK", 1, "blk.1.attn_k.weight", 12),
    ("q4km", "WV", 1, "blk.1.attn_v.weight", 12), ("q4km", "WO", 1, "blk.1.attn_output.weight", 12),
    ("q4km", "GATE", 1, "blk.1.ffn_gate.weight", 12), ("q4km", "UP", 1, "blk.1.ffn_up.weight", 12),
    ("q4km", "DOWN", 1, "blk.1.ffn_down.weight", 12), ("q4km", "GATE", 0, "blk.0.ffn_gate.weight", 14),
    ("q4km", "DOWN", 2, "blk.2.ffn_down.weight", 14), ("q4km", "OUTPUT", 0, "output.weight", 14),
    ("q8_0", "WQ", 0, "blk.0.attn_q.weight", 8), ("q8_0", "DOWN", 1, "blk.1.ffn_down.weight", 8),
    ("q8_0", "OUTPUT", 0, "output.weight", 8), ("f16", "UP", 0, "blk.0.ffn_up.weight", 1),
    ("f16", "WO", 1, "blk.1.attn_output.weight", 1), ("dream", "WK", 1, "blk.1.attn_k.weight", 12),
    ("dream", "OUTPUT", 0, "output.weight", 14), ("wide", "WQ", 0, "blk.0.attn_q.weight", 12),
    ("wide", "GATE", 0, "blk.0.ffn_gate.weight", 14), ("wide", "DOWN", 0, "blk.0.ffn_down.weight", 14),
    ("wide", "OUTPUT", 0, "output.weight", 14),
]


def dequantized(orc, om, tname):
    t, k, n, ptr = om.tensor(tname)
    nbytes = {0: 4 * k, 1: 2 * k, 8: k // 32 * 34, 12: k // 256 * 144, 14: k // 256 * 210}[t] * n
    raw = np.ctypeslib.as_array((C.c_uint8 * nbytes).from_address(ptr))
    return orc.dequantize(raw, t, k * n).reshape(n, k)


@pytest.mark.parametrize("case", GEMM_CASES, ids=lambda c: f"{c[0]}-{c[3]}")
@pytest.mark.parametrize("M", [1, 17, 64, 150, 162, 200, 320, 600])
def test_gemm_parity(pkg, orc, models, case, M):
    """One linear layer against the exact product (f64 on the dequantized weights), within
    GEMM_MEANREL mean relative error; the oracle's f32 GEMM is reported beside it."""
    name, role, layer, tname, gtype = case
    model = pkg.Model(models[name])
    ctx = pkg.Context(model, 0)
    om = orc.OracleModel(models[name])
    assert om.tensor(tname)[0] == gtype
    K = om.tensor(tname)[1]
    x = np.random.default_rng(M).standard_normal((M, K)).astype(np.float32)
    y = ctx.linear(getattr(pkg, role), layer, x)
    exact = x.astype(np.float64) @ dequantized(orc, om, tname).astype(np.float64).T
    mx, rel = metrics(y, exact)
    omx, orel = metrics(om.matmul(tname, x), exact)
    assert rel < GEMM_MEANREL and mx < 2 * GEMM_MEANREL * np.abs(exact).max(), (mx, rel, omx, orel)
    ctx.close(); model.close(); om.close()


@pytest.mark.parametrize("name,n", [("q4km", 80), ("q4km", 320), ("q8_0", 96), ("f16", 64), ("dream", 192),
                                    ("tiny", 40), ("tiny_gqa", 33), ("tied", 48), ("wide", 256), ("wide", 320)])
def test_forward_logits_parity(pkg, orc, models, name, n):
    model = pkg.Model(models[name])
    ctx = pkg.Context(model, 0)
    om = orc.OracleModel(models[name])
    toks = np.random.default_rng(n).integers(0, om.n_vocab - 2, n).astype(np.int32)
    got = ctx.forward(toks)
    ref = om.forward(toks)
    mx, rel = metrics(got, ref)
    scale = max(1.0, float(np.abs(ref).max()))
    print(f"{name} n={n}: max-abs {mx:.3e} (logit scale {scale:.1f}) mean-rel {rel:.3e}")
    # the test-e2e model has N(0,1) weights: logits of size ~30, so max-abs is relative to that scale
    assert rel < LOGIT_MEANREL and mx < LOGIT_MAXABS * scale, (mx, rel)
    # top-1 may differ only between near-tied logits of the reference
    pick = ref[np.arange(n), got.argmax(-1)]
    assert (ref.max(-1) - pick <= 2 * mx + 1e-6).all()
    ctx.close(); model.close(); om.close()


def _teacher_forced(pkg, orc, path, n_prompt, n_gen, params_kw):
    """Run the device loop step by step beside an oracle session fed the device's own
    commits (teacher forcing, the protocol of a divergence-free per-step comparison):
    every step, the oracle runs the reference's full or cached forward on the same
    sequence and cache state, and the device's whole persistent logits buffer and its
    active-row count must match it (diffuse-graph.cpp:395-673, diffuse-cache.h:78-145);
    then the reference sampler, replayed on the device's own logits, must make the
    device's commits bit for bit (diffuse-sampler.cpp:222-323)."""
    model = pkg.Model(path)
    ctx = pkg.Context(model, 0)
    om = orc.OracleModel(path)
    hp = model.hparams
    rng = np.random.default_rng(n_prompt * 7 + n_gen)
    prompt = rng.integers(0, hp.mask_token_id - 1, n_prompt).astype(np.int32)
    P = pkg.SamplerParams(**params_kw)
    OP = orc.SamplerParams(**params_kw)
    sess = orc.OracleSession(om, prompt, n_gen, OP)
    ctx.gen_begin(prompt, n_gen, P)
    n_masked, initialized, near_ties, worst = n_gen, False, 0, (0.0, 0.0)
    for step in range(P.n_steps):
        if n_masked == 0:
            break
        seq = ctx.gen_tokens()
        masked = np.zeros(seq.size, np.uint8)
        masked[n_prompt:] = seq[n_prompt:] == hp.mask_token_id
        force = (not P.use_cache) or (not initialized) or (P.cache_refresh > 0 and step > 0 and step % P.cache_refresh == 0)
        k = pkg.tokens_to_unmask(step, P.n_steps, n_masked, P.schedule)
        st = ctx.gen_step(step, k, force)
        initialized = initialized or bool(P.use_cache)
        n_act = sess.forward(step)
        assert st["n_active"] == n_act, (step, st["n_active"], n_act)
        logits = ctx.logits_rows(0, seq.size)
        mx, rel = metrics(logits, sess.logits())
        scale = max(1.0, float(np.abs(logits).max()))
        assert rel < LOGIT_MEANREL and mx < LOGIT_MAXABS * scale, (step, st["used_cache"], mx, rel)
        worst = max(worst, (rel, mx))
        pos, tok = ctx.gen_commits()
        ref = orc.sampler_step(logits, seq, masked, hp.is_dream, step, OP)
        if P.remasking == 2:
            # Entropy keys are f32 sums of expf terms: the reference adds them serially,
            # the kernel as a tree, so the last bits differ.  The commit sets may then
            # differ only by swaps between candidates whose reference entropies are
            # within EPS of the cut (or of tau, for the early-exit count).
            EPS = 2e-5
            cand = np.flatnonzero(masked)
            H = dict(zip(cand.tolist(), ref["entropy"].tolist()))
            g, r = set(pos.tolist()), set(ref["pos"].tolist())
            if st["n_unmasked"] != ref["n"]:
                near_tau = [h for h in H.values() if abs(h - P.entropy_threshold) < EPS]
                assert near_tau, (st["n_unmasked"], ref["n"])
            if g != r:
                cut = max(H[p] for p in r)
                for p in g ^ r:
                    assert abs(H[p] - cut) < EPS * max(1.0, cut), (p, H[p], cut)
                near_ties += len(g ^ r)
            common = sorted(g & r)
            gt = dict(zip(pos.tolist(), tok.tolist())); rt = dict(zip(ref["pos"].tolist(), ref["tok"].tolist()))
            assert [gt[p] for p in common] == [rt[p] for p in common]
        else:
            assert st["n_unmasked"] == ref["n"]
            np.testing.assert_array_equal(tok, ref["tok"])
            np.testing.assert_array_equal(pos, ref["pos"])
        sess.commit(pos, tok)
        n_masked = st["n_masked"]
    print(f"teacher-forced {params_kw}: worst step logits mean-rel {worst[0]:.2e} max-abs {worst[1]:.2e}")
    out = ctx.gen_tokens()[n_prompt:]
    sess.close(); ctx.close(); model.close(); om.close()
    return out, near_ties


@pytest.mark.parametrize("kw", [
    dict(n_steps=8, remasking=0, use_cache=1),
    dict(n_steps=8, remasking=0, use_cache=0),
    dict(n_steps=8, remasking=4, use_cache=1),
    dict(n_steps=8, remasking=2, use_cache=1, entropy_threshold=0.0),
    dict(n_steps=6, remasking=3, use_cache=1, cache_refresh=3, cache_keep_active=1),
    dict(n_steps=8, remasking=0, use_cache=1, cache_keep_active=2),
], ids=["lowconf-cache", "lowconf-nocache", "margin", "entropy", "maskgit-refresh-keep", "lowconf-keep2"])
def test_sampler_bit_exact_teacher_forced(pkg, orc, models, kw):
    _teacher_forced(pkg, orc, models["q4km"], 16, 32, kw)


def test_dream_shifted_logits_teacher_forced(pkg, orc, models):
    _teacher_forced(pkg, orc, models["dream"], 24, 16, dict(n_steps=8, remasking=2, use_cache=1, entropy_threshold=1.5))


def test_tied_lm_head_teacher_forced(pkg, orc, models):
    # output.weight absent: the lm_head is token_embd (diffuse-model.cpp:157-158)
    _teacher_forced(pkg, orc, models["tied"], 16, 24, dict(n_steps=6, remasking=0, use_cache=1))


def test_temperature_sampling_teacher_forced(pkg, orc, models):
    """temperature > 0 (diffuse-sampler.cpp:256-269), step by step: the host gives the
    device the reference's uniforms (std::mt19937(seed), one std::generate_canonical per
    masked position in position order, orc.canonical); on the device's own logits the
    reference's draw with the same uniform (orc.sample_row) must be the device's committed
    token, unless the uniform lies within EPS of a cumulative sum (device expf and tree
    sums against libm expf and serial sums); the commit set must be the reference's
    top-k by the drawn tokens' probabilities."""
    EPS = 1e-5
    path = models["q4km"]
    model = pkg.Model(path)
    ctx = pkg.Context(model, 0)
    hp = model.hparams
    n_prompt, n_gen, T, seed = 16, 32, 0.8, 5
    prompt = np.random.default_rng(9).integers(0, hp.mask_token_id - 1, n_prompt).astype(np.int32)
    P = pkg.SamplerParams(n_steps=8, remasking=0, use_cache=1, temperature=T, seed=seed)
    U = orc.canonical(seed, n_gen * P.n_steps)
    ctx.gen_begin(prompt, n_gen, P)
    n_masked, initialized, off, checked, near = n_gen, False, 0, 0, 0
    for step in range(P.n_steps):
        if n_masked == 0:
            break
        seq = ctx.gen_tokens()
        cand = np.flatnonzero(seq[n_prompt:] == hp.mask_token_id) + n_prompt
        assert cand.size == n_masked
        force = not initialized
        k = pkg.tokens_to_unmask(step, P.n_steps, n_masked, P.schedule)
        u = U[off:off + n_masked]
        off += n_masked
        ctx.gen_set_uniforms(u)
        st = ctx.gen_step(step, k, force)
        initialized = True
        logits = ctx.logits_rows(0, seq.size)
        pos, tok = ctx.gen_commits()
        draws = {int(p): orc.sample_row(logits[p], T, u[i]) for i, p in enumerate(cand)}
        assert st["n_unmasked"] == k
        step_near = [p for p in cand.tolist() if draws[p][2] < EPS]
        near += len(step_near)
        for p, t in zip(pos.tolist(), tok.tolist()):
            if draws[p][2] >= EPS:
                assert t == draws[p][0], (step, p, t, draws[p])
                checked += 1
        if not step_near:
            # LOW_CONFIDENCE: the k candidates of highest probability (ties within a few ulp may swap)
            conf = {p: d[1] for p, d in draws.items()}
            ranked = sorted(conf, key=lambda p: -conf[p])
            g, r = set(pos.tolist()), set(ranked[:k])
            if g != r:
                cut = conf[ranked[k - 1]]
                for p in g ^ r:
                    assert abs(conf[p] - cut) <= 1e-5 * max(cut, 1e-30), (step, p, conf[p], cut)
        n_masked = st["n_masked"]
    print(f"temperature {T}: {checked} committed draws checked, {near} near a cumulative-sum boundary")
    assert checked >= n_gen - near - 1
    ctx.close(); model.close()


@pytest.mark.parametrize("name,kw", [
    ("q4km", dict(n_steps=8, remasking=0, use_cache=1)),
    ("q4km", dict(n_steps=8, remasking=0, use_cache=1, temperature=0.8, seed=3)),
    ("q4km", dict(n_steps=8, remasking=1, use_cache=1, seed=7)),
    ("dream", dict(n_steps=8, remasking=2, use_cache=1, entropy_threshold=1.5)),
    ("tiny", dict(n_steps=8, remasking=0, use_cache=0)),
], ids=["q4km-lowconf", "q4km-temperature", "q4km-random", "dream-entropy", "tiny-nocache"])
def test_generate_tokens_agree_with_oracle(pkg, orc, models, name, kw):
    """Free-running runs of the whole loop through the public API (diffuse_generate)
    against the oracle's: committed tokens, per-step commit counts, active-row counts and,
    for RANDOM remasking, the committed positions of every step (the host's std::shuffle
    of the candidate list with the shared mt19937, diffuse-sampler.cpp:307)."""
    model = pkg.Model(models[name])
    ctx = pkg.Context(model, 0)
    om = orc.OracleModel(models[name])
    prompt = np.random.default_rng(5).integers(0, om.mask_token_id - 1, 16).astype(np.int32)
    got, info = ctx.generate(prompt, 32, pkg.SamplerParams(**kw), trace=True)
    ref, rtr = om.generate(prompt, 32, orc.SamplerParams(**kw))
    agree = float((got == ref).mean())
    n = info["steps_run"]
    print(f"{name} {kw}: token agreement {agree:.4f}, steps {n}")
    assert (got != om.mask_token_id).all()
    assert agree >= 0.995, agree
    assert n == rtr["steps_run"]
    np.testing.assert_array_equal(info["n_unmasked"][:n], rtr["n_unmask"][:n])
    np.testing.assert_array_equal(info["n_active"][:n], rtr["n_active"][:n])
    if kw["remasking"] == 1:
        np.testing.assert_array_equal(info["commit_pos"][:n], rtr["commit_pos"][:n])
    ctx.close(); model.close(); om.close()


def test_load_errors_are_reported(pkg, tmp_path):
    p = tmp_path / "bad.gguf"
    p.write_bytes(b"GGUF\x03\x00\x00\x00" + b"\x00" * 8)
    with pytest.raises(pkg.DiffuseError):
        pkg.Model(p)
    with pytest.raises(pkg.DiffuseError):
        pkg.Model(tmp_path / "nope.gguf")
