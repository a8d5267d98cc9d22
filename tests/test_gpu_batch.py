"""Several sequences stepped together (one forward per step over all live sequences' active
rows) against the same sequences run alone, and, step by step, against the oracle's
reference loop for each sequence (needs a B200)."""
import numpy as np
import pytest

from conftest import MINI_DREAM, MINI_LLADA, metrics

pytestmark = pytest.mark.gpu

LOGIT_MAXABS, LOGIT_MEANREL = 2e-2, 1e-3


@pytest.fixture(scope="module")
def models(pkg, model_dir):
    return dict(q4km=pkg.synth_model(model_dir / "b_llada.gguf", MINI_LLADA, "q4_k_m", seed=41, n_layer=2),
                dream=pkg.synth_model(model_dir / "b_dream.gguf", MINI_DREAM, "q4_k_m", seed=42, n_layer=2))


def _prompts(hp, lens, seed):
    rng = np.random.default_rng(seed)
    return [rng.integers(0, hp.mask_token_id - 1, n).astype(np.int32) for n in lens]


@pytest.mark.parametrize("name,kw", [
    ("q4km", dict(n_steps=8, remasking=0, use_cache=1)),
    ("q4km", dict(n_steps=8, remasking=1, use_cache=1, seed=3)),
    ("q4km", dict(n_steps=8, remasking=1, use_cache=1, seed=4, temperature=0.9)),
    ("dream", dict(n_steps=8, remasking=2, use_cache=1, entropy_threshold=1.5)),
], ids=["lowconf", "random", "random-temperature", "dream-entropy"])
def test_batch_matches_sequences_run_alone(pkg, models, name, kw):
    model = pkg.Model(models[name])
    ctx = pkg.Context(model, 0)
    prompts = _prompts(model.hparams, [7, 30, 16, 1, 45], 11)
    got, info = ctx.generate_batch(prompts, 24, pkg.SamplerParams(**kw), trace=True)
    for i, pr in enumerate(prompts):
        alone, atr = ctx.generate(pr, 24, pkg.SamplerParams(**kw), trace=True)
        agree = float((got[i] == alone).mean())
        assert agree >= 0.995, (i, agree)
        n = atr["steps_run"]
        np.testing.assert_array_equal(info["n_unmasked"][:n, i], atr["n_unmasked"][:n])
        np.testing.assert_array_equal(info["n_active"][:n, i], atr["n_active"][:n])
    ctx.close(); model.close()


@pytest.mark.parametrize("name,kw,lens", [
    ("q4km", dict(n_steps=6, remasking=0, use_cache=1, cache_keep_active=1), [12, 5, 33]),
    ("dream", dict(n_steps=8, remasking=2, use_cache=1, entropy_threshold=2.5), [20, 9]),
], ids=["llada-keep1", "dream-entropy-early-exit"])
def test_batch_teacher_forced_against_oracle(pkg, orc, models, name, kw, lens):
    """Each sequence of the batch beside its own oracle session, fed the device's commits:
    the sequence's active-row count, its rows of the persistent logits buffer and its
    commits (the reference sampler replayed on the device's logits) must match step by
    step, including sequences whose loop ends early."""
    model = pkg.Model(models[name])
    ctx = pkg.Context(model, 0)
    om = orc.OracleModel(models[name])
    hp = model.hparams
    n_gen = 16
    prompts = _prompts(hp, lens, 5)
    P, OP = pkg.SamplerParams(**kw), orc.SamplerParams(**kw)
    sess = [orc.OracleSession(om, pr, n_gen, OP) for pr in prompts]
    ctx.gen_begin_batch(prompts, n_gen, P)
    offs = np.cumsum([0] + [len(p) + n_gen for p in prompts])
    masked_left = [n_gen] * len(prompts)
    initialized = False
    for step in range(P.n_steps):
        live = [i for i, m in enumerate(masked_left) if m > 0]
        if not live:
            break
        seq_all = ctx.gen_tokens()
        force = (not P.use_cache) or (not initialized)
        sched = [pkg.tokens_to_unmask(step, P.n_steps, m, P.schedule) if m > 0 else -1 for m in masked_left]
        st = ctx.gen_step_batch(step, sched, force)
        initialized = True
        commits = ctx.gen_commits_batch()
        logits_all = ctx.logits_rows(0, int(offs[-1]))
        for i in live:
            a, b = offs[i], offs[i + 1]
            n_act = sess[i].forward(step)
            assert st[i]["n_active"] == n_act, (step, i, st[i]["n_active"], n_act)
            lg = logits_all[a:b]
            mx, rel = metrics(lg, sess[i].logits())
            assert rel < LOGIT_MEANREL and mx < LOGIT_MAXABS * max(1.0, float(np.abs(lg).max())), (step, i, mx, rel)
            seq = seq_all[a:b]
            masked = np.zeros(seq.size, np.uint8)
            masked[len(prompts[i]):] = seq[len(prompts[i]):] == hp.mask_token_id
            ref = orc.sampler_step(lg, seq, masked, hp.is_dream, step, OP)
            pos, tok = commits[i]
            if P.remasking == 2:
                # serial vs tree entropy sums: swaps only between near-equal entropies
                g, r = set((pos - a).tolist()), set(ref["pos"].tolist())
                assert len(g ^ r) <= 2, (step, i, g ^ r)
            else:
                np.testing.assert_array_equal(pos - a, ref["pos"])
                np.testing.assert_array_equal(tok, ref["tok"])
            sess[i].commit(pos - a, tok)
            masked_left[i] = st[i]["n_masked"]
    for s in sess:
        s.close()
    ctx.close(); model.close(); om.close()
