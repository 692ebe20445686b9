"""The tensor-parallel partition of the host model (jd_tp_shard_of, the shards that
jdg_host_upload_tp uploads) checked on CPU ranks over gloo: every rank runs the host forward
(janusdoe.c:3160-3322) on its shard only — its query/KV heads, its Wo contraction columns,
its FFN hidden slice (gate/up rows, down columns), its vocabulary rows — with the oracle's
packed row kernels, all-reduces the Wo and down outputs, adds the replicated LoRA
parliament once on the reduced residual, and gathers the vocabulary slices.  The result
must equal the unsplit oracle forward: logits within 1e-4 (norm-relative) and the same
elections and EMA per layer."""
import ctypes as C
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CASES = {
    # arch, dim, layers, heads, kv heads, ffn, vocab, dtype, theta, lora rank, alive adapters
    "q8_neox": ("qwen2", 256, 2, 8, 4, 512, 1000, 8, 1e4, 8, 4),
    "q4k_norm": ("llama", 1024, 2, 8, 4, 2048, 1000, 12, 5e5, 16, 8),
}
STEPS = [(11, 0), (407, 1), (93, 2), (5, 3)]   # (token, position) fed in order


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _row_bytes(dt, cols):
    return {0: cols * 4, 8: cols // 32 * 34, 12: cols // 256 * 144}[dt]


def _block(dt):
    return {0: 1, 8: 32, 12: 256}[dt]


def _packed(ptr, dt, rows, cols):
    rb = _row_bytes(dt, cols)
    return np.frombuffer(C.string_at(ptr, rows * rb), np.uint8).reshape(rows, rb)


def _cols(W, dt, c0, c1):
    """Columns [c0, c1) of packed rows (whole blocks)."""
    bb = _row_bytes(dt, _block(dt))
    return np.ascontiguousarray(W[:, c0 // _block(dt) * bb: c1 // _block(dt) * bb])


def _rms(x, w, eps):
    D = x.size
    ss = np.add.accumulate((x * x).astype(np.float32), dtype=np.float32)[-1]
    inv = np.float32(1.0) / np.sqrt(np.float32(ss / np.float32(D) + np.float32(eps)))
    return (x * inv * w).astype(np.float32) if w is not None else (x * inv).astype(np.float32)


def _rope(v, pos, theta, HD, norm):
    half = HD // 2
    out = v.copy()
    for h in range(v.size // HD):
        for i in range(half):
            ang = np.float32(pos) / np.float32(np.power(np.float32(theta), np.float32(2.0 * i / HD), dtype=np.float32))
            co, si = np.cos(ang, dtype=np.float32), np.sin(ang, dtype=np.float32)
            a, b = (2 * i, 2 * i + 1) if norm else (i, i + half)
            x0, x1 = v[h * HD + a], v[h * HD + b]
            out[h * HD + a] = x0 * co - x1 * si
            out[h * HD + b] = x0 * si + x1 * co
    return out


def _worker(rank, world, port, path, case, q):
    import sys
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import conftest  # noqa: F401
    import janus_doe_b200 as jd
    from oracle.oracle import JdoElect, MAXE, Oracle
    from oracle.oracle import HostModel as OHost
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        arch, D, L, Hn, KVH, FF, V, dt, theta, R, na = CASES[case]
        orc = Oracle()
        orc.lib.jdo_set_threads(1)
        om = OHost(orc, path, R, -1, 16)
        om.lora_seed(19, na, 0.01, 1.0 / D ** 0.5)
        hm = jd.HostModel(path, lora_rank=R)
        sh = jd.JdTpShard()
        jd.check(jd.lib().jd_tp_shard_of(C.byref(hm.h), rank, world, C.byref(sh)))
        hm.close()
        h = om.h
        HD, HG = D // Hn, Hn // KVH
        q0, nq = sh.q_head0 * HD, sh.q_heads * HD
        k0, nk = sh.kv_head0 * HD, sh.kv_heads * HD
        f0, nf = sh.hidden0, sh.hidden
        kd, qd = KVH * HD, Hn * HD
        W = []
        for l in range(L):
            ly = h.layers[l]
            W.append(dict(
                q=np.ascontiguousarray(_packed(ly.wq, ly.wq_dt, qd, D)[q0:q0 + nq]),
                k=np.ascontiguousarray(_packed(ly.wk, ly.wk_dt, kd, D)[k0:k0 + nk]),
                v=np.ascontiguousarray(_packed(ly.wv, ly.wv_dt, kd, D)[k0:k0 + nk]),
                o=_cols(_packed(ly.wo, ly.wo_dt, D, qd), ly.wo_dt, q0, q0 + nq),
                g=np.ascontiguousarray(_packed(ly.gate, ly.gate_dt, FF, D)[f0:f0 + nf]),
                u=np.ascontiguousarray(_packed(ly.up, ly.up_dt, FF, D)[f0:f0 + nf]),
                d=_cols(_packed(ly.down, ly.down_dt, D, FF), ly.down_dt, f0, f0 + nf),
                an=np.ctypeslib.as_array(ly.attn_norm, (D,)).copy() if ly.attn_norm else None,
                fn=np.ctypeslib.as_array(ly.ffn_norm, (D,)).copy() if ly.ffn_norm else None,
                dts=(ly.wq_dt, ly.wo_dt, ly.gate_dt, ly.down_dt)))
        out_w = np.ascontiguousarray(_packed(h.output, h.output_dt, V, D)[sh.vocab0:sh.vocab0 + sh.vocab])
        onorm = np.ctypeslib.as_array(h.output_norm, (D,)).copy() if h.output_norm else None
        emb = np.ctypeslib.as_array(h.tok_emb, (V, D))
        kc = np.zeros((L, 16, nk), np.float32)
        vc = np.zeros((L, 16, nk), np.float32)
        cons = np.full(32, 0.5, np.float32)
        tr = (JdoElect * 32)()
        mv = orc.qmatvec
        results = []
        for tok, pos in STEPS:
            x = emb[tok].copy()
            trace = []
            for l in range(L):
                w = W[l]
                xn = _rms(x, w["an"], h.rms_eps)
                qv = _rope(mv(w["q"], w["dts"][0], xn, nq, D), pos, theta, HD, h.rope_norm)
                kv = _rope(mv(w["k"], w["dts"][0], xn, nk, D), pos, theta, HD, h.rope_norm)
                vv = mv(w["v"], w["dts"][0], xn, nk, D)
                kc[l, pos], vc[l, pos] = kv, vv
                ao_in = np.zeros(nq, np.float32)
                for j in range(sh.q_heads):
                    g = (sh.q_head0 + j) // HG - sh.kv_head0     # local KV head of global query head
                    qh = qv[j * HD:(j + 1) * HD]
                    s = np.array([np.float32(np.dot(qh, kc[l, t, g * HD:(g + 1) * HD]))
                                  * np.float32(1.0 / np.sqrt(np.float32(HD))) for t in range(pos + 1)], np.float32)
                    e = np.exp(s - s.max()).astype(np.float32)
                    a = (e / e.sum(dtype=np.float32)).astype(np.float32)
                    ao_in[j * HD:(j + 1) * HD] = (a[:, None] * vc[l, :pos + 1, g * HD:(g + 1) * HD]).sum(0)
                ao = torch.from_numpy(mv(w["o"], w["dts"][1], ao_in, D, nq))
                dist.all_reduce(ao)                                # row-parallel Wo: partial sums
                x = (x + ao.numpy()).astype(np.float32)
                fnx = _rms(x, w["fn"], h.rms_eps)
                gt = mv(w["g"], w["dts"][2], fnx, nf, D)
                up = mv(w["u"], w["dts"][2], fnx, nf, D)
                hh = (gt / (np.float32(1) + np.exp(-gt)) * up).astype(np.float32)
                fo = torch.from_numpy(mv(w["d"], w["dts"][3], hh, D, nf))
                dist.all_reduce(fo)                                # row-parallel down
                x = (x + fo.numpy() * np.float32(h.layer_focus[l])).astype(np.float32)
                # the parliament is replicated: same input xn on every rank, delta added once
                sel = (C.c_int * MAXE)()
                wts = (C.c_float * MAXE)()
                xp = np.ascontiguousarray(xn, np.float32)
                cp = cons[l:].ctypes.data_as(C.POINTER(C.c_float))
                kk = orc.lib.jdo_host_elect(C.byref(h), l, cp, xp.ctypes.data_as(C.POINTER(C.c_float)),
                                            D, sel, wts, C.byref(tr[l]))
                for ki in range(kk):
                    ex = sel[ki]
                    A = np.ctypeslib.as_array(h.A[l][ex], (D, R))
                    Bm = np.ctypeslib.as_array(h.B[l][ex], (R, D))
                    t = (Bm @ xn.astype(np.float64)).astype(np.float32)
                    x = (x + np.float32(h.lora_alpha * wts[ki]) * (A.astype(np.float64) @ t).astype(np.float32)).astype(np.float32)
                trace.append((kk, [sel[i] for i in range(kk)], float(cons[l])))
            xo = _rms(x, onorm, h.rms_eps)
            lg = torch.from_numpy(mv(out_w, h.output_dt, xo, sh.vocab, D)) if sh.vocab else torch.zeros(0)
            per = (V + world - 1) // world
            pad = torch.zeros(per, dtype=torch.float32)
            pad[:lg.numel()] = lg
            parts = [torch.zeros(per, dtype=torch.float32) for _ in range(world)]
            dist.all_gather(parts, pad)                            # vocabulary-parallel LM head
            results.append((torch.cat(parts)[:V].numpy(), trace))
        om.close()
        q.put((rank, (sh.q_head0, sh.q_heads, sh.kv_head0, sh.kv_heads, sh.hidden0, sh.hidden, sh.vocab0, sh.vocab),
               results if rank == 0 else None))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("case", sorted(CASES))
def test_tp_shards_match_unsplit_oracle(jd, orc, tmp_path, case, world):
    arch, D, L, Hn, KVH, FF, V, dt, theta, R, na = CASES[case]
    path = str(tmp_path / ("%s.gguf" % case))
    jd.write_synthetic_gguf(path, arch, L, D, FF, Hn, KVH, V, theta, 1e-5, dt, 23, 0.02)
    from oracle.oracle import HostModel as OHost
    om = OHost(orc, path, R, -1, 16)
    om.lora_seed(19, na, 0.01, 1.0 / D ** 0.5)
    ref = [om.forward(t, p, trace=True) for t, p in STEPS]
    om.close()
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, path, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=280) for _ in range(world)], key=lambda t: t[0])
    for p in procs:
        p.join(timeout=30)
        assert p.exitcode == 0
    shards = [r[1] for r in res]
    # the shards tile the model: heads, KV heads, hidden units, vocabulary
    assert sum(s[1] for s in shards) == Hn and sum(s[3] for s in shards) == KVH
    assert sum(s[5] for s in shards) == FF and sum(s[7] for s in shards) == V
    assert [s[0] for s in shards] == [sum(t[1] for t in shards[:i]) for i in range(world)]
    for (lg, trace), (lo, tro) in zip(res[0][2], ref):
        err = float(np.max(np.abs(lg - lo)) / np.max(np.abs(lo)))
        assert err <= 1e-4, err
        for l in range(L):
            k, sel, ema = trace[l]
            assert k == int(tro["k"][l]) and sel == list(tro["sel"][l][:k]), (l, k, sel)
            assert abs(ema - float(tro["ema"][l])) <= 1e-6
