"""Hebbian --learn on the GPU (jdg_host_learn) against the oracle's restatement of
host_learn_run (itself pinned to the reference build): after a pass over a token stream the
LoRA factors of every expert agree within 1e-3 of their scale, the alive flags, the RNG state
and the notorch offset are equal, and the next forward's logits and elections agree.

The tolerance is the logits' (1e-3): every update is scaled by the prophecy-debt signal,
which takes the difference of the best and the next token's logits, so a logit difference
of 1e-6 (f32 summation order) can move the signal, and the updates, by up to ~1e-4 when the
two logits are close."""
import numpy as np
import pytest

from _util import LOGIT_TOL, compare_trace, logit_err
from oracle.oracle import HostModel as OHost

pytestmark = pytest.mark.gpu

CASES = {
    # arch, dim, layers, heads, kv, ffn, vocab, dtype, theta, lora rank, adapters, lr, passes
    "q8_r8": ("qwen2", 256, 2, 4, 2, 512, 800, 8, 1e4, 8, 4, 0.05, 1),
    "q4k_r16": ("llama", 512, 2, 8, 2, 1024, 1200, 12, 5e5, 16, 8, 0.5, 1),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_learn_matches_oracle(jd, orc, gpu_ctx, tmp_path, name):
    arch, D, L, H, KV, FF, V, dt, theta, R, na, lr, passes = CASES[name]
    path = str(tmp_path / ("%s.gguf" % name))
    jd.write_synthetic_gguf(path, arch, L, D, FF, H, KV, V, theta, 1e-5, dt, 41, 0.02)
    hm = jd.HostModel(path, lora_rank=R)
    hm.lora_seed(7, na, 0.01, 1.0 / D ** 0.5)
    om = OHost(orc, path, R, -1, 64)
    om.lora_seed(7, na, 0.01, 1.0 / D ** 0.5)
    eng = jd.Engine.host(gpu_ctx, hm, 1, 64)
    try:
        toks = np.random.default_rng(11).integers(0, V, 20).astype(np.int32)
        rng_g = rng_o = 42
        off_g = off_o = 0
        for _ in range(passes):
            dg, rng_g, off_g = eng.host_learn(toks, lr, rng_g, off_g)
            do, rng_o, off_o = om.learn(toks, lr, rng_o, off_o)
            assert (dg, rng_g, off_g) == (do, rng_o, off_o)
        moved = 0.0
        for l in range(L):
            for e in range(16):
                A, B, al = eng.expert(l, e, D, R)
                Ao, Bo, alo = om.expert(l, e)
                assert al == alo, (l, e)
                if Ao is None or not alo:
                    continue
                scale = max(float(np.abs(Ao).max()), float(np.abs(Bo).max()))
                assert float(np.abs(A - Ao).max()) <= 1e-3 * scale, (l, e)
                assert float(np.abs(B - Bo).max()) <= 1e-3 * scale, (l, e)
                moved = max(moved, scale)
        assert moved > 0
        # the learned parliament in the next decode
        eng.reset()
        om.reset()
        for pos, t in enumerate(toks[:6]):
            lo, tro = om.forward(int(t), pos, trace=True)
            _, _, lg, tr = eng.step([int(t)], [pos], logits=True, trace=True)
            assert logit_err(lg[0], lo) <= LOGIT_TOL, pos
            assert not compare_trace(tr, tro, L), pos
    finally:
        eng.close()
        om.close()
        hm.close()
