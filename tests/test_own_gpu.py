"""Own-model decode on the GPU against the oracle (parity tests proper, through the C ABI).

Workloads are the synthetic configs: depth-4 (dim 256, 4 experts, vocab 2256), depth-8
(dim 512, GQA 8/4, 6 experts, vocab 4256), depth-12 (dim 768, 12/4 heads, 8 experts with
5-8 alive per layer, vocab 8256, context 1024).  Weights are N(0, 0.02) from the seed.
"""
import numpy as np
import pytest

from _util import LOGIT_TOL, compare_trace, compare_trace_ties, greedy_near_tie, logit_err
from oracle.oracle import OwnModel

pytestmark = pytest.mark.gpu


@pytest.fixture(params=["step", "chain", "generic"])
def b1_path(request, monkeypatch):
    """Batch 1 runs the persistent one-kernel step (JDG_B1=step), the PDL kernel chain
    (JDG_B1=chain) or the generic batched kernels (JDG_GENERIC=1)."""
    monkeypatch.delenv("JDG_GENERIC", raising=False)
    monkeypatch.setenv("JDG_B1", "chain")
    if request.param == "generic":
        monkeypatch.setenv("JDG_GENERIC", "1")
    elif request.param == "step":
        monkeypatch.setenv("JDG_B1", "step")
    return request.param


def _pair(jd, orc, depth, seed, masks=False, **over):
    cfg_o = orc.config(depth, **over)
    om = OwnModel(orc, cfg_o, seed, 0.02, masks)
    pm = jd.Model.seeded(jd.config_from_depth(depth, **over), seed, 0.02, masks)
    for l in range(cfg_o.depth):
        assert pm.alive(l) == om.alive(l)
    return om, pm


def _teacher_forced(om, eng, stream, n_prompt, check_from=0):
    """Feed the oracle's greedy stream to both; compare logits, elections and picks."""
    L = om.c.depth
    worst, ties, flips = 0.0, 0, []
    for pos in range(len(stream) - 1):
        t = stream[pos]
        lo, tro = om.forward(t, pos, trace=True)
        nxt, _, lg, trg = eng.step([t], [pos], logits=True, trace=True)
        if pos < check_from:
            continue
        err = logit_err(lg[0], lo)
        worst = max(worst, err)
        assert err <= LOGIT_TOL, "pos %d logit err %.3g" % (pos, err)
        bad = compare_trace(trg, tro, L)
        assert not bad, "pos %d election mismatch %s" % (pos, bad[:3])
        if pos + 1 >= n_prompt:
            if int(nxt[0]) != int(np.argmax(lo)):
                if greedy_near_tie(lo):
                    ties += 1
                else:
                    flips.append(pos)
    assert not flips, "greedy flips at %s" % flips
    return worst, ties


def _oracle_greedy(om, prompt, n_gen):
    om.reset()
    stream = list(int(t) for t in prompt)
    pos = 0
    lg = None
    for t in prompt:
        lg = om.forward(t, pos)
        pos += 1
    for _ in range(n_gen):
        nxt = int(np.argmax(lg))
        stream.append(nxt)
        lg = om.forward(nxt, pos)
        pos += 1
    om.reset()
    return stream


def test_depth4_greedy_full(jd, orc, gpu_ctx, b1_path):
    """depth-4, seed 0, 32-token prompt + 128 greedy tokens at batch 1."""
    om, pm = _pair(jd, orc, 4, 0, vocab_size=2256, seq_len=256)
    prompt, _ = orc.prompt(0 * 1000 + 0, 2256, 32)
    stream = _oracle_greedy(om, prompt, 128)
    eng = jd.Engine.own(gpu_ctx, pm, 1)
    try:
        worst, ties = _teacher_forced(om, eng, stream, 32)
        # free-running device loop: prompt fed on device, then 128 greedy tokens
        eng.reset()
        eng.set_prompt(np.array([prompt]), [32])
        eng.run(1, 31 + 128)
        hist = eng.history(1, 128)[0]
        assert list(hist) == stream[32:], "free-running stream differs"
        assert eng.launches() > 0
    finally:
        eng.close()
        om.close()


def test_depth12_masks_greedy(jd, orc, gpu_ctx, b1_path):
    """depth-12 variable topology (5-8 alive experts per layer), GQA 12/4, ctx 1024."""
    om, pm = _pair(jd, orc, 12, 3, True, n_kv_heads=4, vocab_size=8256, seq_len=1024)
    n_alive = [sum(om.alive(l)) for l in range(12)]
    assert min(n_alive) >= 5 and max(n_alive) <= 8
    prompt, _ = orc.prompt(3 * 1000 + 0, 8256, 40)
    stream = _oracle_greedy(om, prompt, 40)
    eng = jd.Engine.own(gpu_ctx, pm, 1)
    try:
        _teacher_forced(om, eng, stream, 40)
        eng.reset()
        eng.set_prompt(np.array([prompt]), [40])
        eng.run(1, 39 + 40)
        assert list(eng.history(1, 40)[0]) == stream[40:]
    finally:
        eng.close()
        om.close()


def test_long_context_attention(jd, orc, gpu_ctx, b1_path):
    """Attention over ~1000 positions (16 chunks of the split-K kernel) on a depth-4 model."""
    om, pm = _pair(jd, orc, 4, 7, vocab_size=2256, seq_len=1024)
    prompt, _ = orc.prompt(7 * 1000 + 1, 2256, 1000)
    eng = jd.Engine.own(gpu_ctx, pm, 1)
    try:
        eng.reset()
        eng.set_prompt(np.array([prompt]), [1000])
        eng.run(1, 999)            # positions 0..998 on the device
        om.reset()
        for pos in range(999):
            om.forward(prompt[pos], pos)
        lo, tro = om.forward(prompt[999], 999, trace=True)
        nxt, _, lg, trg = eng.step([prompt[999]], [999], logits=True, trace=True)
        assert logit_err(lg[0], lo) <= LOGIT_TOL
        assert not compare_trace(trg, tro, 4)
    finally:
        eng.close()
        om.close()


@pytest.mark.parametrize("B", [2, 5, 33])
def test_batched_teacher_forced(jd, orc, gpu_ctx, B):
    """depth-8 GQA model, B independent sequences through the grouped-expert GEMM path."""
    depth, V = 8, 4256
    om, pm = _pair(jd, orc, depth, 1, vocab_size=V, seq_len=256)
    eng = jd.Engine.own(gpu_ctx, pm, B)
    try:
        P, G = 6, 6
        prompts = [orc.prompt(1 * 1000 + s, V, P)[0] for s in range(B)]
        # oracle streams, one sequence after another (own EMA state per sequence)
        streams, logits, traces = [], [], []
        for s in range(B):
            om.reset()
            st, lgs, trs = list(int(t) for t in prompts[s]), [], []
            for pos in range(P + G - 1):
                lo, tro = om.forward(st[pos], pos, trace=True)
                lgs.append(lo)
                trs.append(tro)
                if pos + 1 >= P:
                    st.append(int(np.argmax(lo)))
            streams.append(st)
            logits.append(lgs)
            traces.append(trs)
        eng.reset()
        for pos in range(P + G - 1):
            tok = np.array([streams[s][pos] for s in range(B)], np.int32)
            nxt, _, lg, trg = eng.step(tok, np.full(B, pos, np.int32), logits=True, trace=True)
            for s in range(B):
                assert logit_err(lg[s], logits[s][pos]) <= LOGIT_TOL, (s, pos)
                assert not compare_trace(trg, traces[s][pos], depth, b=s), (s, pos)
    finally:
        eng.close()
        om.close()


def test_sampling_matches_oracle(jd, orc, gpu_ctx):
    """temperature 0.8, top-k 40 sampling (chat settings) with per-sequence xorshift states:
    with the oracle's token stream forced, the GPU's sampled token equals the oracle's
    sample() of the oracle's logits with the same RNG state at >= 95% of steps, and the
    RNG states advance identically."""
    depth, V, B = 8, 4256, 4
    om, pm = _pair(jd, orc, depth, 1, vocab_size=V, seq_len=256)
    eng = jd.Engine.own(gpu_ctx, pm, B)
    eng.set_sampling(0.8, 40)
    try:
        P, G = 4, 12
        agree = total = 0
        states = []
        streams = []
        for s in range(B):
            pr, st = orc.prompt(1 * 1000 + s, V, P)
            streams.append(list(int(t) for t in pr))
            states.append(st)
        lgs_by_seq = [[] for _ in range(B)]
        for s in range(B):
            om.reset()
            st = states[s]
            for pos in range(P + G - 1):
                lo = om.forward(streams[s][pos], pos)
                if pos + 1 >= P:
                    r, st = orc.sample(lo, 0.8, 40, st)
                    streams[s].append(r)
                lgs_by_seq[s].append(lo)
        eng.reset()
        rng = np.array(states, np.uint64)
        for pos in range(P + G - 1):
            tok = np.array([streams[s][pos] for s in range(B)], np.int32)
            r_in = rng.copy()
            nxt, rng_out, lg, _ = eng.step(tok, np.full(B, pos, np.int32), rng=r_in, logits=True)
            if pos + 1 >= P:
                for s in range(B):
                    exp_tok, exp_state = orc.sample(lgs_by_seq[s][pos], 0.8, 40, int(rng[s]))
                    assert int(rng_out[s]) == exp_state
                    total += 1
                    agree += int(int(nxt[s]) == int(streams[s][pos + 1]))
                rng = rng_out
        assert total > 0 and agree / total >= 0.95, (agree, total)
    finally:
        eng.close()
        om.close()


@pytest.mark.parametrize("P", [2, 37, 200])
def test_batched_prefill_matches_token_by_token(jd, orc, gpu_ctx, P):
    """Batched prompt prefill (all prompt tokens as one batch per layer, EMA as an ordered
    scan) on the depth-12 variable-topology model: every prompt token's k, elected experts,
    weights and EMA per layer equal the oracle's token-by-token decode, and the greedy stream
    that follows (the KV cache the prefill wrote) equals the oracle's."""
    om, pm = _pair(jd, orc, 12, 3, True, n_kv_heads=4, vocab_size=8256, seq_len=1024)
    prompt, _ = orc.prompt(3 * 1000 + 7, 8256, P)
    G = 24
    om.reset()
    traces, lg = [], None
    for pos, t in enumerate(prompt):
        lg, tr = om.forward(int(t), pos, trace=True)
        traces.append(tr)
    exp = []
    pos = P
    for _ in range(G):
        nxt = int(np.argmax(lg))
        exp.append(nxt)
        lg = om.forward(nxt, pos)
        pos += 1
    eng = jd.Engine.own(gpu_ctx, pm, 1)
    try:
        eng.reset()
        eng.set_prompt(np.array([prompt]), [P])
        ms = eng.prefill(1)
        assert ms > 0
        tok, p = eng.state(1)
        assert int(p[0]) == P - 1 and int(tok[0]) == int(prompt[-1])
        tr = eng.prefill_trace(P - 1)
        ties = []
        for t in range(P - 1):
            bad, tie = compare_trace_ties(tr, traces[t], 12, b=t)
            assert not bad, (t, bad[:3])
            if tie:             # a reference near-tie: the residual streams part here
                ties.append((t, tie))
                break
        print("prefill P=%d: near-ties %s" % (P, ties))
        eng.run(1, G)   # the last prompt token, then greedy tokens
        if not ties:
            assert list(eng.history(1, G)[0]) == exp
    finally:
        eng.close()
        om.close()
