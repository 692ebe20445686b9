"""The oracle against the golden fixtures that the reference produced (tests/golden/).

These run on CPU without the reference build; tests/golden/gen_golden.py regenerates the
fixtures from the reference source.  The oracle restates the reference in its operation
order, so every comparison here is exact.
"""
import ctypes as C
import hashlib
import os

import numpy as np
import pytest

from oracle.oracle import HostModel, OwnModel, fptr

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return np.load(os.path.join(GOLD, name))


def test_rng_streams(orc):
    g = load("rng.npz")
    for i, s in enumerate(g["states"]):
        st = C.c_uint64(int(s))
        assert [orc.lib.jdo_rng_next(C.byref(st)) for _ in range(64)] == [int(v) for v in g["next"][i]]
        st = C.c_uint64(int(s))
        u = np.array([orc.lib.jdo_rand_uniform(C.byref(st)) for _ in range(64)], np.float32)
        assert np.array_equal(u, g["uniform"][i])
        st = C.c_uint64(int(s))
        n = np.array([orc.lib.jdo_rand_normal(C.byref(st)) for _ in range(64)], np.float32)
        assert np.array_equal(n, g["normal"][i])


def test_f16_all_values(orc):
    bits = load("f16.npz")["bits"]
    got = np.array([orc.lib.jdo_f16_to_f32(h) for h in range(65536)], np.float32).view(np.uint32)
    assert np.array_equal(got, bits)


@pytest.mark.parametrize("dt", [1, 2, 6, 8, 12, 14])
def test_quant_kernels(orc, dt):
    g = load("quant.npz")
    W, x, y, dq = g["W%d" % dt], g["x%d" % dt], g["y%d" % dt], g["dq%d" % dt]
    rows, cols = W.shape[0], 512
    assert np.array_equal(orc.qmatvec(W, dt, x, rows, cols), y)
    assert np.array_equal(orc.dequant(W, rows * cols, dt), dq)


def test_sample(orc):
    g = load("sample.npz")
    for i in range(len(g["pick"])):
        r, st = orc.sample(g["logits"][i], float(g["temp"][i]), int(g["topk"][i]), int(g["state"][i]))
        assert r == int(g["pick"][i]) and st == int(g["state_after"][i]), i


@pytest.mark.parametrize("name", ["own_depth4", "own_depth12"])
def test_own_decode(orc, name):
    g = load("%s.npz" % name)
    depth, kv, V, ctx, seed, masks, P, G = [int(v) for v in g["cfg"]]
    over = dict(vocab_size=V, seq_len=ctx)
    if kv:
        over["n_kv_heads"] = kv
    m = OwnModel(orc, orc.config(depth, **over), seed, 0.02, bool(masks))
    try:
        assert np.array_equal(np.array([m.alive(l) for l in range(depth)], np.int32), g["alive"])
        toks = list(g["tokens"][:P])
        keep = {int(p): i for i, p in enumerate(g["logit_pos"])}
        for pos in range(P + G - 1):
            lg = m.forward(toks[pos], pos)
            assert np.array_equal(m.ema(), g["ema"][pos]), pos
            if pos in keep:
                assert np.array_equal(lg, g["logits"][keep[pos]]), pos
            if pos + 1 >= P:
                toks.append(int(np.argmax(lg)))
        assert toks == list(g["tokens"])
    finally:
        m.close()


@pytest.mark.parametrize("name", ["host_q8", "host_q4k"])
def test_host_decode(orc, jd, tmp_path, name):
    from golden.gen_golden import HOST
    g = load("%s.npz" % name)
    arch, D, L, H, KV, FF, V, dt, theta, R, na = HOST[name]
    path = str(tmp_path / "h.gguf")
    jd.write_synthetic_gguf(path, arch, L, D, FF, H, KV, V, theta, 1e-5, dt, 7, 0.02)
    assert hashlib.md5(open(path, "rb").read()).hexdigest() == str(g["gguf_md5"])
    hm = HostModel(orc, path, R, -1, 64)
    hm.lora_seed(11, na, 0.01, 1.0 / D ** 0.5)
    try:
        for pos, t in enumerate(g["tokens"]):
            lg = hm.forward(int(t), pos)
            assert np.array_equal(lg, g["logits"][pos]), pos
            assert np.array_equal(hm.ema(), g["ema"][pos]), pos
    finally:
        hm.close()


def test_host_tokenizer_golden(jd, tmp_path):
    """The library's tokenizer and token printing against the reference's outputs recorded
    in host_tokens.npz (no reference build needed)."""
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "host_tokens.npz"), allow_pickle=True)
    path = str(tmp_path / "tok.gguf")
    jd.write_synthetic_gguf(path, "llama", 1, 256, 512, 4, 2, 3000, 1e4, 1e-5, 8, 3, 0.02)
    assert hashlib.md5(open(path, "rb").read()).hexdigest() == str(g["gguf_md5"])
    hm = jd.HostModel(path, lora_rank=8)
    try:
        off = 0
        for t, n in zip(g["texts"], g["lens"]):
            assert hm.tokenize(bytes(t), 256) == [int(x) for x in g["ids"][off:off + n]], bytes(t)[:40]
            off += n
        for i, s in zip(range(-2, 3003), g["printed"]):
            assert hm.token_text(i) == bytes(s), i
    finally:
        hm.close()
