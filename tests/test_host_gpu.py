"""Host GGUF decode (`--host` path) on the GPU against the oracle, through the C ABI.

Synthetic llama-family GGUFs are written by the library's generator (weights N(0, 0.02)
quantised per block), loaded by the product loader (GPU side) and by the oracle's own
loader; the LoRA parliament is drawn from the same seed on both sides.
"""
import os

import numpy as np
import pytest

from _util import LOGIT_TOL, compare_trace, greedy_near_tie, logit_err
from oracle.oracle import HostModel as OHost

pytestmark = pytest.mark.gpu

SMALL = {
    # name: arch, dim, layers, heads, kv, ffn, vocab, dtype, theta, lora rank, alive adapters
    "q8_neox": ("qwen2", 256, 2, 4, 2, 512, 1000, 8, 1e4, 8, 4),
    "q4k_norm": ("llama", 512, 3, 4, 2, 1024, 2000, 12, 5e5, 16, 8),
    "q8_gqa8": ("qwen2", 512, 2, 8, 1, 1024, 1500, 8, 1e4, 8, 4),
}
# full-width layers of the 1.1B Q8_0 and 8B Q4_K shapes (fewer layers, smaller vocabulary):
# rows of 5632 and 14336 weights exercise the widest register buckets of the batch-1 chain
# output heads and layers in the other GGUF types the loader keeps packed
MIXED = {
    # name: arch, dim, layers, heads, kv, ffn, vocab, layer dtype, head dtype, theta, lora rank, adapters
    "q4k_q6k_head": ("llama", 512, 2, 8, 2, 1024, 2000, 12, 14, 5e5, 16, 8),
    "q4_0_f16_head": ("qwen2", 256, 2, 4, 2, 512, 1000, 2, 1, 1e4, 8, 4),
    "q5_0_q6k_head": ("llama", 512, 2, 8, 4, 1024, 1500, 6, 14, 5e5, 8, 4),
}
WIDE = {
    "q8_c4_layer": ("qwen2", 2048, 2, 32, 4, 5632, 3000, 8, 1e4, 8, 4),
    "q4k_c5_layer": ("llama", 4096, 1, 32, 8, 14336, 2000, 12, 5e5, 16, 8),
}


@pytest.fixture(params=["chain", "generic"])
def b1_path(request, monkeypatch):
    """Batch 1 runs either the PDL kernel chain (default) or the generic kernels."""
    if request.param == "generic":
        monkeypatch.setenv("JDG_GENERIC", "1")
    else:
        monkeypatch.delenv("JDG_GENERIC", raising=False)
    return request.param


def _models(jd, orc, name, tmp_path, max_seq=96):
    arch, D, L, H, KV, FF, V, dt, theta, R, na = SMALL[name] if name in SMALL else WIDE[name]
    path = str(tmp_path / ("%s.gguf" % name))
    jd.write_synthetic_gguf(path, arch, L, D, FF, H, KV, V, theta, 1e-5, dt, 17, 0.02)
    hm = jd.HostModel(path, lora_rank=R)
    hm.lora_seed(23, na, 0.01, 1.0 / D ** 0.5)
    om = OHost(orc, path, R, -1, max_seq)
    om.lora_seed(23, na, 0.01, 1.0 / D ** 0.5)
    return hm, om, V


@pytest.mark.parametrize("dt,rows,cols", [(8, 300, 2048), (8, 64, 5632), (12, 200, 4096), (12, 96, 1792), (0, 50, 512)])
@pytest.mark.parametrize("B", [1, 3, 40])
def test_qmatvec_matches_oracle(jd, orc, gpu_ctx, dt, rows, cols, B):
    """Packed GEMV (B=1) and GEMM (B>1; Q4_K on the tensor cores, 32 tokens per launch)
    against jd_qmatvec's restatement."""
    if B > 1 and cols % 256:
        pytest.skip("batched path needs 256-multiples")
    if B > 3 and dt != 12:
        pytest.skip("the 40-token case exercises the tensor-core GEMM")
    rng = np.random.default_rng(rows + cols + dt)
    if dt == 0:
        W = rng.standard_normal((rows, cols)).astype(np.float32) * 0.02
        Wb = W.view(np.uint8).reshape(rows, -1)
    else:
        # build packed rows through the synthetic writer's quantiser via a tiny GGUF
        Wb = _random_packed(rng, dt, rows, cols)
    x = rng.standard_normal((B, cols)).astype(np.float32)
    got = jd.qmatvec(gpu_ctx, Wb, dt, x, rows, cols)
    for b in range(B):
        if dt == 0:
            ref = (W.astype(np.float64) @ x[b].astype(np.float64)).astype(np.float32)
        else:
            ref = orc.qmatvec(Wb, dt, x[b], rows, cols)
        err = np.max(np.abs(got[b] - ref)) / max(1e-30, np.max(np.abs(ref)))
        assert err <= 1e-5, (b, err)


def _random_packed(rng, dt, rows, cols):
    """Random but well-formed packed rows: finite f16 scales, random codes."""
    if dt == 8:
        nb = cols // 32
        blk = np.zeros((rows, nb, 34), np.uint8)
        d = (rng.random((rows, nb)) * 1e-3 + 1e-4).astype(np.float16)
        blk[:, :, 0:2] = d.view(np.uint8).reshape(rows, nb, 2)
        blk[:, :, 2:] = rng.integers(-127, 128, (rows, nb, 32)).astype(np.int8).view(np.uint8)
        return blk.reshape(rows, -1)
    nb = cols // 256
    blk = rng.integers(0, 256, (rows, nb, 144)).astype(np.uint8)
    d = (rng.random((rows, nb)) * 1e-3 + 1e-4).astype(np.float16)
    dm = (rng.random((rows, nb)) * 1e-3).astype(np.float16)
    blk[:, :, 0:2] = d.view(np.uint8).reshape(rows, nb, 2)
    blk[:, :, 2:4] = dm.view(np.uint8).reshape(rows, nb, 2)
    return blk.reshape(rows, -1)


def test_qmatvec_rejects_unsupported(jd, gpu_ctx):
    """Packed dtypes without a kernel (here Q5_K, type 13) are reported, never read as f32
    (janusdoe.c:2739)."""
    W = np.zeros((4, 176), np.uint8)
    with pytest.raises(jd.JdError) as ei:
        jd.qmatvec(gpu_ctx, W, 13, np.zeros(256, np.float32), 4, 256)
    assert ei.value.code == jd.JD_EUNSUPPORTED


@pytest.mark.parametrize("dt,rows,cols", [(14, 300, 2048), (14, 70, 4096), (2, 200, 1024), (6, 130, 2048),
                                          (1, 90, 512)])
@pytest.mark.parametrize("B", [1, 3])
def test_qmatvec_more_types(jd, orc, gpu_ctx, dt, rows, cols, B):
    """Q6_K (native 6-bit kernels), Q4_0 / Q5_0 (int8 codes in the Q8_0 layout) and F16 (as
    f32) against jd_qmatvec's restatement, on rows written by the library's quantiser."""
    rng = np.random.default_rng(rows + dt)
    x = rng.standard_normal((B, cols)).astype(np.float32)
    Wb = _typed_rows(jd, dt, rows, cols, rows + cols)
    got = jd.qmatvec(gpu_ctx, Wb, dt, x, rows, cols)
    for b in range(B):
        ref = orc.qmatvec(Wb, dt, x[b], rows, cols)
        err = np.max(np.abs(got[b] - ref)) / max(1e-30, np.max(np.abs(ref)))
        assert err <= 1e-5, (b, err)


def _typed_rows(jd, dt, rows, cols, seed):
    """rows x cols weights of type dt: the output head of a synthetic GGUF in that type."""
    import tempfile
    from oracle.oracle import Oracle
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "t.gguf")
        jd.write_synthetic_gguf(path, "llama", 1, cols, 256, cols // 64, cols // 64, rows, 1e4, 1e-5, 8, seed, 0.02,
                                out_dtype=dt)
        hm = jd.HostModel(path, lora_rank=8)
        try:
            assert hm.h.output_dt == dt
            import ctypes as C
            rb = {1: cols * 2, 2: cols // 32 * 18, 6: cols // 32 * 22, 14: cols // 256 * 210}[dt]
            return np.frombuffer(C.string_at(hm.h.output, rows * rb), np.uint8).reshape(rows, rb).copy()
        finally:
            hm.close()


def _oracle_stream(om, prompt, n_gen):
    om.reset()
    st, lgs, trs = list(int(t) for t in prompt), [], []
    for pos in range(len(prompt) + n_gen - 1):
        lo, tro = om.forward(st[pos], pos, trace=True)
        lgs.append(lo)
        trs.append(tro)
        if pos + 1 >= len(prompt):
            st.append(int(np.argmax(lo)))
    return st, lgs, trs


@pytest.mark.parametrize("name", sorted(SMALL) + sorted(WIDE))
def test_host_greedy_parity(jd, orc, gpu_ctx, tmp_path, name, b1_path):
    """Teacher-forced logits/elections, then the free-running device loop's greedy stream."""
    hm, om, V = _models(jd, orc, name, tmp_path)
    L = hm.h.n_layers
    P, G = (12, 24) if name in SMALL else (5, 6)
    prompt = np.random.default_rng(5).integers(0, V, P).astype(np.int32)
    stream, lgs, trs = _oracle_stream(om, prompt, G)
    eng = jd.Engine.host(gpu_ctx, hm, 1, 96)
    try:
        eng.reset()
        for pos in range(P + G - 1):
            nxt, _, lg, tr = eng.step([stream[pos]], [pos], logits=True, trace=True)
            assert logit_err(lg[0], lgs[pos]) <= LOGIT_TOL, (pos, logit_err(lg[0], lgs[pos]))
            bad = compare_trace(tr, trs[pos], L)
            assert not bad, (pos, bad)
            if pos + 1 >= P and int(nxt[0]) != stream[pos + 1]:
                assert greedy_near_tie(lgs[pos]), pos
        eng.reset()
        eng.set_prompt(prompt[None, :], [P])
        eng.run(1, P - 1 + G)
        assert list(eng.history(1, G)[0]) == stream[P:]
    finally:
        eng.close()
        om.close()
        hm.close()


def test_host_batched_parity(jd, orc, gpu_ctx, tmp_path):
    """Several independent sequences (own KV and EMA each) through the batched GEMM path."""
    hm, om, V = _models(jd, orc, "q4k_norm", tmp_path)
    L = hm.h.n_layers
    B, P, G = 5, 6, 6
    prompts = np.random.default_rng(9).integers(0, V, (B, P)).astype(np.int32)
    ref = [_oracle_stream(om, prompts[b], G) for b in range(B)]
    eng = jd.Engine.host(gpu_ctx, hm, B, 96)
    try:
        eng.reset()
        for pos in range(P + G - 1):
            tok = np.array([ref[b][0][pos] for b in range(B)], np.int32)
            nxt, _, lg, tr = eng.step(tok, np.full(B, pos, np.int32), logits=True, trace=True)
            for b in range(B):
                assert logit_err(lg[b], ref[b][1][pos]) <= LOGIT_TOL, (b, pos)
                assert not compare_trace(tr, ref[b][2][pos], L, b=b), (b, pos)
    finally:
        eng.close()
        om.close()
        hm.close()


def test_host_batched_parity_wide(jd, orc, gpu_ctx, tmp_path):
    """A full 32-sequence tile of the 8B Q4_K layer shape (dim 4096, ffn 14336): every slot of
    the tensor-core GEMM's token tile, the batched prep and the batched parliament."""
    hm, om, V = _models(jd, orc, "q4k_c5_layer", tmp_path)
    L = hm.h.n_layers
    B, P, G = 32, 3, 2
    prompts = np.random.default_rng(11).integers(0, V, (B, P)).astype(np.int32)
    ref = [_oracle_stream(om, prompts[b], G) for b in range(B)]
    eng = jd.Engine.host(gpu_ctx, hm, B, 96)
    try:
        eng.reset()
        for pos in range(P + G - 1):
            tok = np.array([ref[b][0][pos] for b in range(B)], np.int32)
            nxt, _, lg, tr = eng.step(tok, np.full(B, pos, np.int32), logits=True, trace=True)
            for b in range(B):
                assert logit_err(lg[b], ref[b][1][pos]) <= LOGIT_TOL, (b, pos)
                assert not compare_trace(tr, ref[b][2][pos], L, b=b), (b, pos)
    finally:
        eng.close()
        om.close()
        hm.close()


def test_host_lora_sidecar_roundtrip(jd, orc, gpu_ctx, tmp_path):
    """A LoRA parliament saved to the sidecar and loaded back gives identical logits."""
    hm, om, V = _models(jd, orc, "q8_neox", tmp_path)
    side = str(tmp_path / "lora.bin")
    hm.lora_save(side)
    arch, D, L, H, KV, FF, V, dt, theta, R, na = SMALL["q8_neox"]
    hm2 = jd.HostModel(str(tmp_path / "q8_neox.gguf"), lora_rank=R)
    hm2.lora_load(side)
    e1 = jd.Engine.host(gpu_ctx, hm, 1, 32)
    e2 = jd.Engine.host(gpu_ctx, hm2, 1, 32)
    try:
        for pos, t in enumerate([3, 14, 15, 92]):
            _, _, l1, _ = e1.step([t], [pos], logits=True)
            _, _, l2, _ = e2.step([t], [pos], logits=True)
            assert np.array_equal(l1, l2)
    finally:
        e1.close()
        e2.close()
        om.close()
        hm.close()
        hm2.close()


@pytest.mark.parametrize("name", sorted(MIXED))
def test_host_mixed_types_parity(jd, orc, gpu_ctx, tmp_path, name, b1_path):
    """Host models whose layers are Q4_K / Q4_0 / Q5_0 with a Q6_K or F16 output head, kept
    packed: teacher-forced logits and elections at batch 1 and at 3 sequences."""
    arch, D, L, H, KV, FF, V, dt, odt, theta, R, na = MIXED[name]
    path = str(tmp_path / ("%s.gguf" % name))
    jd.write_synthetic_gguf(path, arch, L, D, FF, H, KV, V, theta, 1e-5, dt, 31, 0.02, out_dtype=odt)
    hm = jd.HostModel(path, lora_rank=R)
    assert hm.h.output_dt == odt and hm.h.layers[0].wq_dt == dt
    hm.lora_seed(23, na, 0.01, 1.0 / D ** 0.5)
    om = OHost(orc, path, R, -1, 64)
    om.lora_seed(23, na, 0.01, 1.0 / D ** 0.5)
    try:
        for B in (1, 3):
            P, G = 4, 4
            prompts = np.random.default_rng(B).integers(0, V, (B, P)).astype(np.int32)
            ref = [_oracle_stream(om, prompts[b], G) for b in range(B)]
            eng = jd.Engine.host(gpu_ctx, hm, B, 64)
            try:
                eng.reset()
                for pos in range(P + G - 1):
                    tok = np.array([ref[b][0][pos] for b in range(B)], np.int32)
                    nxt, _, lg, tr = eng.step(tok, np.full(B, pos, np.int32), logits=True, trace=True)
                    for b in range(B):
                        assert logit_err(lg[b], ref[b][1][pos]) <= LOGIT_TOL, (B, b, pos)
                        assert not compare_trace(tr, ref[b][2][pos], L, b=b), (B, b, pos)
            finally:
                eng.close()
    finally:
        om.close()
        hm.close()
