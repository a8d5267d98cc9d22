"""The benchmark's work accounting (no GPU): the active rows per denoising step of config 2
follow the reference's cached loop with the tokens_to_unmask counts, and the algorithmic
FLOPs of one generation are the 45.90 TFLOP the roofline divides by."""
import importlib.util
import pathlib
import sys

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("dfb_bench", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules["dfb_bench"] = mod
    spec.loader.exec_module(mod)
    return mod


def test_c2_active_rows_follow_the_cached_loop(bench, pkg):
    cfg = bench.CONFIGS["c2"]
    rows = bench.c2_active_rows(cfg)
    # step 0 is the full forward over prompt + block; step s > 0 recomputes the masked
    # positions plus the ones committed at step s - 1 (diffuse-cache.h update timing)
    counts, masked = [], cfg["block"]
    for s in range(cfg["steps"]):
        k = pkg.tokens_to_unmask(s, cfg["steps"], masked, 0)
        counts.append(k)
        masked -= k
    expect = [cfg["prompt"] + cfg["block"]]
    left = cfg["block"]
    for s in range(1, cfg["steps"]):
        left -= counts[s - 1]
        expect.append(left + counts[s - 1])
    assert rows == expect
    assert rows == [320, 256, 255, 251, 245, 237, 226, 213, 198, 181, 162, 142, 120, 97, 74, 50]


def test_c2_algorithmic_flops(bench, pkg):
    cfg = bench.CONFIGS["c2"]
    hp = type("HP", (), dict(n_embd=4096, n_ff=12288, n_vocab=126464, n_layer=32, n_head=32, n_head_kv=32))
    flops = bench.c2_algorithmic_flops(hp, bench.c2_active_rows(cfg), cfg["prompt"] + cfg["block"])
    assert abs(flops / 1e12 - 45.90) < 0.01
    # step 0 alone (320 rows, full forward) is 4.852 TFLOP
    f0 = bench.c2_algorithmic_flops(hp, [320], 320)
    assert abs(f0 / 1e12 - 4.852) < 0.002


def test_reference_arm_runs_the_oracle_only(bench, tmp_path, monkeypatch, capsys):
    """`bench.py --impl reference` on a two-layer architecture of the same family: one JSON
    line whose bench step is the timed sample (two full-depth denoising steps) and whose
    generation time is extrapolated, with no product library loaded on that path."""
    import json
    import types
    monkeypatch.setitem(bench.ARCH, "tiny", dict(is_dream=0, n_vocab=512, n_embd=256, n_head=4, n_head_kv=4,
                                                 n_layer=2, n_ff=512, n_ctx=512, mask_token_id=500,
                                                 rope_theta=10000.0, rms_norm_eps=1e-5, with_bias=0))
    monkeypatch.setenv("DFB_BENCH_DIR", str(tmp_path))
    cfg = dict(bench.CONFIGS["c2"], arch="tiny", desc="tiny")
    loaded_before = set(sys.modules)
    assert bench.run_reference(types.SimpleNamespace(steps=2, warmup=1, gpus=1, config="c2"), cfg) == 0
    line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["extrapolated"] is True
    assert line["value"] > 0 and line["e2e"]["value"] == line["value"]
    assert 0 < line["ms_per_step"] < line["extrapolated_ms_per_generation"]
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    # the product package (its ctypes bindings of libdfb_cuda / libdiffuse) was not imported here
    assert not any(m.startswith("diffuse_b200") for m in set(sys.modules) - loaded_before)
