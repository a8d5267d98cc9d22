"""The oracle and the host codecs against gguf-py's golden vectors (CPU only)."""
import pathlib

import numpy as np
import pytest

GOLD = np.load(pathlib.Path(__file__).with_name("golden") / "quant_golden.npz")
TYPES = {"q4k": 12, "q6k": 14, "q80": 8}


@pytest.mark.parametrize("name", ["q4k", "q6k", "q80"])
def test_oracle_dequant_matches_gguf_py(orc, name):
    got = orc.dequantize(GOLD[f"{name}_blocks"], TYPES[name], GOLD[f"{name}_values"].size)
    np.testing.assert_array_equal(got, GOLD[f"{name}_values"])


@pytest.mark.parametrize("name", ["q4k", "q6k", "q80"])
def test_host_dequant_matches_gguf_py(pkg, name):
    got = pkg.dequantize_rows(GOLD[f"{name}_blocks"], TYPES[name], GOLD[f"{name}_values"].size)
    np.testing.assert_array_equal(got, GOLD[f"{name}_values"])


def test_host_q8_0_quantizer_bit_exact(pkg):
    got = pkg.quantize_rows(GOLD["q80_src"], 8)
    np.testing.assert_array_equal(got, GOLD["q80_quant"])


@pytest.mark.parametrize("qtype,tol", [(12, 0.08), (14, 0.02), (8, 0.01)])
def test_host_kquant_roundtrip(pkg, qtype, tol):
    rng = np.random.default_rng(1)
    x = (rng.standard_normal(256 * 64) * 0.02).astype(np.float32)
    raw = pkg.quantize_rows(x, qtype)
    y = pkg.dequantize_rows(raw, qtype, x.size)
    rel = np.sqrt(np.mean((x - y) ** 2)) / np.sqrt(np.mean(x ** 2))
    assert rel < tol, rel


def test_schedule_counts_match_reference_formula(pkg, orc):
    # cfg2: B = 256, 16 steps, cosine, every step runs
    n = 256
    counts = []
    for s in range(16):
        k = orc.tokens_to_unmask(s, 16, n, 0)
        assert k == pkg.tokens_to_unmask(s, 16, n, 0)
        counts.append(k)
        n -= k
    assert counts == [1, 4, 6, 8, 11, 13, 15, 17, 19, 20, 22, 23, 23, 24, 25, 25]
    assert n == 0
    for steps in (1, 7, 32):
        for masked in (1, 3, 64, 255):
            for sched in (0, 1):
                for s in range(steps):
                    assert orc.tokens_to_unmask(s, steps, masked, sched) == pkg.tokens_to_unmask(s, steps, masked, sched)


def test_entropy_reference_formula(orc):
    rng = np.random.default_rng(3)
    row = (rng.standard_normal(5000) * 3).astype(np.float32)
    z = row.astype(np.float64) - row.max()
    p = np.exp(z) / np.exp(z).sum()
    ref = float(-(p[p > 1e-10] * np.log(p[p > 1e-10])).sum())
    assert abs(orc.entropy(row) - ref) < 1e-4


def test_temperature_draw_restatement_matches_discrete_distribution(orc):
    """orc_sample_row (the temperature > 0 draw with its uniform given) and orc_canonical
    (std::generate_canonical<double, 53> on std::mt19937) against the oracle's own
    sampling loop, which calls std::discrete_distribution on the rng directly
    (diffuse-sampler.cpp:256-269): the committed tokens and every candidate's confidence
    must agree bit for bit."""
    rng = np.random.default_rng(3)
    V, n_prompt, n = 3000, 8, 24
    total = n_prompt + n
    logits = (rng.standard_normal((total, V)) * 3).astype(np.float32)
    seq = np.zeros(total, np.int32)
    masked = np.zeros(total, np.uint8)
    masked[n_prompt:] = 1
    for T in (0.7, 1.0, 2.5):
        P = orc.SamplerParams(n_steps=4, temperature=T, remasking=0, seed=11)
        ref = orc.sampler_step(logits, seq, masked, False, 0, P)
        u = orc.canonical(11, n)
        cand = np.flatnonzero(masked)
        picks = {}
        for i, p in enumerate(cand):
            k, conf, margin = orc.sample_row(logits[p], T, u[i])
            assert conf == ref["conf"][i], (T, i)
            assert margin >= 0.0
            picks[int(p)] = k
        assert ref["n"] > 0
        for p, t in zip(ref["pos"].tolist(), ref["tok"].tolist()):
            assert picks[p] == t, (T, p)
