"""Pin the oracle against the reference itself (oracle/_ref, built from the reference source
by `make -C oracle ref`).  Skipped where that build is absent.

Every comparison is exact: the restatement follows the reference's operation order and both
are compiled with the same flags.
"""
import os

import numpy as np
import pytest

from oracle.oracle import HostModel, OwnModel, Reference

REF_DIR = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref")
pytestmark = pytest.mark.skipif(not os.path.exists(os.path.join(REF_DIR, "libjdref.so")),
                                reason="reference build (oracle/_ref) not present")


@pytest.fixture(scope="module")
def ref():
    return Reference("")


@pytest.mark.parametrize("depth,over,seed,masks,steps", [
    (2, dict(vocab_size=300, seq_len=64), 11, False, 20),
    (4, dict(vocab_size=2256, seq_len=256), 5, True, 24),
    (8, dict(n_kv_heads=4, vocab_size=4256, seq_len=128), 1, True, 10),
])
def test_own_forward_bit_exact(orc, ref, depth, over, seed, masks, steps):
    ref.own_setup(depth, over.get("n_kv_heads", 0), over["vocab_size"], over["seq_len"], seed, 0.02, masks)
    m = OwnModel(orc, orc.config(depth, **over), seed, 0.02, masks)
    try:
        for l in range(depth):
            assert ref.own_alive(l) == m.alive(l)
        ref.own_reset()
        toks = list(orc.prompt(seed * 1000, over["vocab_size"], 6)[0])
        for pos in range(steps):
            lr, er = ref.own_forward(toks[pos], pos)
            lo = m.forward(toks[pos], pos)
            assert np.array_equal(lr, lo), pos
            assert np.array_equal(er, m.ema()), pos
            if pos + 1 >= len(toks):
                toks.append(int(np.argmax(lr)))
    finally:
        m.close()


def test_sample_bit_exact(orc, ref):
    rng = np.random.default_rng(3)
    for i in range(200):
        V = int(rng.integers(2, 600))
        lg = (rng.standard_normal(V) * rng.uniform(0.1, 5)).astype(np.float32)
        if i % 7 == 0:
            lg[rng.integers(0, V, 5)] = lg.max()  # ties at the top
        temp = float(rng.choice([0.0, 0.3, 0.8, 1.0, 2.0]))
        topk = int(rng.choice([0, 1, 5, 40, V, V + 3]))
        st = int(rng.integers(1, 2 ** 63))
        assert ref.sample(lg, temp, topk, st) == orc.sample(lg, temp, topk, st), i


@pytest.mark.parametrize("dt", [1, 2, 6, 8, 12, 14])
def test_qmatvec_bit_exact(orc, ref, dt):
    from golden.gen_golden import random_packed
    rng = np.random.default_rng(dt)
    for rows, cols in [(3, 256), (17, 1024), (5, 2048)]:
        W = random_packed(rng, dt, rows, cols)
        x = rng.standard_normal(cols).astype(np.float32)
        assert np.array_equal(ref.qmatvec(W, dt, x, rows, cols), orc.qmatvec(W, dt, x, rows, cols))


@pytest.mark.parametrize("arch,dt,rank,variant", [("qwen2", 8, 8, "_r8"), ("llama", 12, 16, ""), ("mistral", 8, 16, "")])
def test_host_forward_bit_exact(orc, jd, tmp_path, arch, dt, rank, variant):
    D, L, H, KV, FF, V = 512, 2, 8, 2, 1024, 700
    path = str(tmp_path / "h.gguf")
    jd.write_synthetic_gguf(path, arch, L, D, FF, H, KV, V, 1e4, 1e-6, dt, 3, 0.02)
    r = Reference(variant)
    r.host_load(path)
    r.lib.jdr_host_lora_seed(9, 6, 0.01, 0.05)
    r.lib.jdr_host_reset_seq(40)
    hm = HostModel(orc, path, rank, -1, 40)
    hm.lora_seed(9, 6, 0.01, 0.05)
    try:
        assert list(r.hdims[:8]) == [hm.h.n_layers, hm.h.dim, hm.h.hidden, hm.h.n_heads, hm.h.n_kv_heads,
                                     hm.h.head_dim, hm.h.vocab, hm.h.rope_norm]
        for pos, t in enumerate(np.random.default_rng(1).integers(0, V, 12)):
            lr, er = r.host_forward(int(t), pos)
            lo = hm.forward(int(t), pos)
            assert np.array_equal(lr, lo) and np.array_equal(er, hm.ema()), pos
    finally:
        r.lib.jdr_host_free()
        hm.close()


def test_own_gguf_export_identical(jd, ref, tmp_path):
    """The library's export_gguf writes the reference's bytes; each loads the other's file."""
    ref.own_setup(4, 0, 2256, 256, 2, 0.02, True)
    a, b = str(tmp_path / "ref.gguf"), str(tmp_path / "lib.gguf")
    ref.lib.jdr_own_export(a.encode())
    m = jd.Model.seeded(jd.config_from_depth(4, vocab_size=2256, seq_len=256), 2, 0.02, True)
    m.export_gguf(b)
    assert open(a, "rb").read() == open(b, "rb").read()
    assert ref.lib.jdr_own_load(b.encode()) == 1
    m2 = jd.Model(jd.config_from_depth(4, vocab_size=2256, seq_len=256))
    m2.load_gguf(a)
    assert all(m2.alive(l) == m.alive(l) for l in range(4))


def test_loaders_reject_truncated(orc, jd, tmp_path):
    path = str(tmp_path / "h.gguf")
    jd.write_synthetic_gguf(path, "llama", 1, 256, 256, 4, 4, 300, 1e4, 1e-6, 8, 3, 0.02)
    data = open(path, "rb").read()
    r = Reference("")
    for cut in (10, 100, len(data) // 2, len(data) - 1):
        bad = str(tmp_path / ("t%d.gguf" % cut))
        open(bad, "wb").write(data[:cut])
        assert r.lib.jdr_host_load(bad.encode(), -1) == 0
        with pytest.raises(ValueError):
            HostModel(orc, bad, 16)
        with pytest.raises(jd.JdError):
            jd.HostModel(bad)


def test_host_learn_matches_reference(jd, orc, tmp_path):
    """The oracle's Hebbian --learn pass (notorch steps on the elected experts, prophecy-debt
    signal, RMS cap, quarantine; janusdoe.c:3091-3147, 3416-3447) equals the reference's
    host_learn_run bit for bit: every expert's A and B, alive flags, RNG state and offset."""
    from oracle.oracle import HostModel as OHost, Reference
    path = str(tmp_path / "learn.gguf")
    jd.write_synthetic_gguf(path, "llama", 2, 256, 512, 4, 2, 500, 1e4, 1e-5, 8, 9, 0.02)
    ref = Reference("")
    ref.host_load(path)
    ref.lib.jdr_host_lora_seed(5, 4, 0.01, 1.0 / 16)
    om = OHost(orc, path, 16, -1, 64)
    om.lora_seed(5, 4, 0.01, 1.0 / 16)
    try:
        toks = np.random.default_rng(3).integers(0, 500, 24).astype(np.int32)
        for lr, rounds in ((0.05, 2), (3.0, 1)):
            for _ in range(rounds):
                got = om.learn(toks, lr, 42, 1)
                exp = ref.host_learn(toks, 64, lr, 42, 1)
                assert got == exp, (got, exp)
                for l in range(2):
                    for e in range(16):
                        a1, b1, al1 = om.expert(l, e)
                        a2, b2, al2 = ref.host_expert(l, e)
                        assert al1 == al2, (l, e)
                        if a1 is not None:
                            assert np.array_equal(a1, a2) and np.array_equal(b1, b2), (l, e)
    finally:
        om.close()
        ref.lib.jdr_host_free()
