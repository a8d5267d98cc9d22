"""The drop-in boundary, proven with the reference's own callers: its command-line tools and
its C++ API test compile unchanged against include/diffuse.h and link against this
repository's libdiffuse.so / libdfb_cuda.so (the reference's include/diffuse.h:71-91
contract); test-forward's model-free checks (the API's defaults) then run on the CPU.
Needs a diffuse-cpp checkout: set DIFFUSE_CPP_CHECKOUT to its root (skipped otherwise)."""
import os
import pathlib
import subprocess

import pytest

REF = os.environ.get("DIFFUSE_CPP_CHECKOUT")
ROOT = pathlib.Path(__file__).resolve().parents[1]
LIB = ROOT / "diffuse-cpp_b200" / "lib"
CALLERS = ["tools/main-cli.cpp", "tools/main-bench.cpp", "tools/dump-logits.cpp", "tests/test-forward.cpp"]


def _build(src: pathlib.Path, out: pathlib.Path):
    cmd = ["g++", "-std=c++17", "-O1", f"-I{ROOT / 'include'}", str(src), f"-L{LIB}", "-ldiffuse", "-ldfb_cuda",
           f"-Wl,-rpath,{LIB}", "-o", str(out)]
    return subprocess.run(cmd, capture_output=True, text=True)


@pytest.mark.skipif(not REF, reason="set DIFFUSE_CPP_CHECKOUT to a diffuse-cpp checkout")
@pytest.mark.parametrize("src", CALLERS)
def test_reference_caller_builds_against_this_library(pkg, tmp_path, src):
    path = pathlib.Path(REF) / src
    assert path.exists(), path
    out = tmp_path / path.stem
    r = _build(path, out)
    assert r.returncode == 0, r.stderr[-2000:]
    assert out.exists()


@pytest.mark.skipif(not REF, reason="set DIFFUSE_CPP_CHECKOUT to a diffuse-cpp checkout")
def test_reference_api_test_runs_its_model_free_checks(pkg, tmp_path):
    out = tmp_path / "test-forward"
    r = _build(pathlib.Path(REF) / "tests/test-forward.cpp", out)
    assert r.returncode == 0, r.stderr[-2000:]
    run = subprocess.run([str(out)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stderr[-2000:]
    for check in ("hparams defaults", "sampler params defaults", "API compilation check"):
        assert f"PASS: {check}" in run.stderr
