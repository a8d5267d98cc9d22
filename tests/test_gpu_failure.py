"""Failure detection on the device, tested without a GPU fault (needs a B200).

Every wait of the dequant GEMM is bounded; when one runs out the kernel raises its error
flag, every CTA gives up, and the host returns DFB_ERR_TIMEOUT instead of hanging.  The
test makes a wait run out on purpose through dfb_debug_stalled_linear: one split-tile
arrival counter starts at a value the tile's contributors can never bring to their count,
and the launch's wait limit is 20 ms.  Nothing traps, faults or hangs; the context must
then compute the same layer exactly as before.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import MINI_LLADA

pytestmark = pytest.mark.gpu

DFB_ERR_TIMEOUT = -5


@pytest.fixture(scope="module")
def mini(pkg, tmp_path_factory):
    return pkg.synth_model(tmp_path_factory.mktemp("fail") / "m.gguf", MINI_LLADA, "q4_k_m", seed=31, n_layer=2)


def test_bounded_wait_times_out_and_context_recovers(pkg, mini):
    model = pkg.Model(mini)
    ctx = pkg.Context(model, 0)
    dfb, _ = pkg.native()
    # ffn_down: 1024 output rows (4 pair tiles) x 11 k-blocks -> every tile split over 11 CTA pairs
    x = np.random.default_rng(3).standard_normal((17, MINI_LLADA["n_ff"])).astype(np.float32)
    before = ctx.linear(pkg.DOWN, 1, x)
    y = np.zeros_like(before)
    rc = dfb.dfb_debug_stalled_linear(ctx.engine, pkg.DOWN, 1, x.ctypes.data_as(C.c_void_p), x.shape[0],
                                      y.ctypes.data_as(C.c_void_p), 20_000_000)
    assert rc == DFB_ERR_TIMEOUT, (rc, dfb.dfb_last_error())
    msg = dfb.dfb_last_error().decode()
    assert "contributors" in msg, msg
    after = ctx.linear(pkg.DOWN, 1, x)
    np.testing.assert_array_equal(after, before)
    toks = np.arange(40, dtype=np.int32)
    assert np.isfinite(ctx.forward(toks)).all()
    ctx.close()
    model.close()
