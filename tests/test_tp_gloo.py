"""Tensor-parallel decomposition (diffuse-cpp_b200/tp.py) on the CPU: the shard plan's split
rules, the cross-rank combination of sampler statistics, and a two-rank gloo execution of the
sharded forward (all-reduce after the output and down projections, vocab-parallel lm_head)
against the unsharded forward and the oracle."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from conftest import TINY, load_package, write_tiny_gguf


def test_plan_split_rules(pkg):
    tp = pkg.tp
    # LLaDA-8B: 32/32 heads x 128, FFN 12288 (48 super-blocks), vocab 126464
    for world in (1, 2, 4, 8):
        shards = tp.plan(32, 32, 128, 12288, 126464, world)
        assert [len(s.heads) for s in shards] == [32 // world] * world
        assert sum(len(s.ff) for s in shards) == 12288 and sum(len(s.vocab) for s in shards) == 126464
    # Dream-7B: 28/4 heads, FFN 18944 = 74 super-blocks: only 2-way
    tp.plan(28, 4, 128, 18944, 152064, 2)
    with pytest.raises(ValueError, match="cuts"):
        tp.plan(28, 4, 128, 18944, 152064, 4)
    with pytest.raises(ValueError, match="heads"):
        tp.plan(28, 4, 128, 18944, 152064, 8)
    # Q8_0 blocks of 32 allow the 4-way Dream FFN split
    tp.plan(28, 4, 128, 18944, 152064, 4, block=32)


def test_combine_stats_matches_whole_rows(pkg):
    tp = pkg.tp
    rng = np.random.default_rng(5)
    z = rng.standard_normal((7, 96)) * 3
    z[0, 10] = z[0, 70] = z[0].max() + 1.0  # tie across slices: the lower index wins
    z[1, 40] = z[1, 41] = z[1].max() + 1.0  # tie inside one slice
    parts = [tp.row_stats(z[:, a:a + 24]) for a in range(0, 96, 24)]
    best, tok, second, ent = tp.combine_stats(parts, [0, 24, 48, 72])
    p = np.exp(z - z.max(axis=1, keepdims=True))
    p /= p.sum(axis=1, keepdims=True)
    for r in range(len(z)):
        order = np.argsort(-z[r], kind="stable")
        assert best[r] == z[r, order[0]] and tok[r] == order[0]
        assert second[r] == z[r, order[1]]
        assert abs(ent[r] - float(-(p[r] * np.log(p[r])).sum())) < 1e-9
    assert tok[0] == 10 and second[0] == best[0] and tok[1] == 40


def _weights(path):
    import gguf
    r = gguf.GGUFReader(str(path))
    W = {}
    for t in r.tensors:
        ne = [int(x) for x in t.shape]
        a = np.asarray(t.data, dtype=np.float64)
        W[t.name] = a.reshape(ne[1], ne[0]) if len(ne) == 2 else a.reshape(ne[0])
    return W


HP = dict(n_embd=TINY["hidden"], n_head=TINY["heads"], n_head_kv=2, n_layer=TINY["layers"], n_ff=TINY["ff"],
          n_vocab=TINY["vocab"], rope_theta=500000.0, rms_norm_eps=1e-5)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, path, tokens, out_q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    import torch
    pkg = load_package()
    dp = pkg.dp.DataParallel.from_env(timeout_s=60, backend="gloo")
    W = _weights(path)
    hd = HP["n_embd"] // HP["n_head"]
    shard = pkg.tp.plan(HP["n_head"], HP["n_head_kv"], hd, HP["n_ff"], HP["n_vocab"], world, block=1)[rank]

    def allreduce(a):
        t = torch.from_numpy(np.ascontiguousarray(a))
        dp._dist.all_reduce(t)
        return t.numpy()
    logits = pkg.tp.forward_rank(W, HP, np.asarray(tokens), shard, allreduce)
    stats = pkg.tp.row_stats(logits)
    out_q.put((rank, logits, stats, shard.vocab.start))
    dp.close()


def test_two_rank_forward_matches_unsharded_and_oracle(pkg, orc, tmp_path):
    path = write_tiny_gguf(tmp_path / "tiny_tp.gguf", kv_heads=2, bias=True, dream=False)
    tokens = np.random.default_rng(9).integers(0, 200, 24).tolist()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port, world = _free_port(), 2
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, path, tokens, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict((r[0], r[1:]) for r in (q.get(timeout=120) for _ in range(world)))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    tp_logits = np.concatenate([res[r][0] for r in range(world)], axis=1)

    W = _weights(path)
    hd = HP["n_embd"] // HP["n_head"]
    full = pkg.tp.forward_rank(W, HP, np.asarray(tokens), pkg.tp.plan(HP["n_head"], HP["n_head_kv"], hd, HP["n_ff"],
                                                                       HP["n_vocab"], 1, block=1)[0], lambda a: a)
    assert np.abs(tp_logits - full).max() < 1e-9 * max(1.0, np.abs(full).max())

    # the unsharded numpy forward is the reference graph: agrees with the oracle (f32)
    om = orc.OracleModel(path)
    ref = om.forward(np.asarray(tokens, np.int32))
    om.close()
    err = np.abs(full - ref).sum() / np.abs(ref).sum()
    assert err < 1e-4, err

    # sampler statistics combined across the vocab slices = statistics of the whole rows
    best, tok, second, ent = pkg.tp.combine_stats([res[r][1] for r in range(world)], [res[r][2] for r in range(world)])
    whole = pkg.tp.row_stats(full)
    assert np.array_equal(tok, whole[:, 1].astype(np.int64))
    assert np.allclose(best, whole[:, 0]) and np.allclose(second, whole[:, 2])
