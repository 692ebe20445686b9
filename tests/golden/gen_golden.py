"""Generate the golden fixtures in this directory from the reference itself.

Runs the reference source compiled by oracle/Makefile (oracle/_ref/libjdref*.so, built with
`make -C oracle ref`) and records its outputs for fixed seeds:
  rng.npz      xorshift64 stream, rand_uniform, rand_normal from fixed states
  f16.npz      jd_f16_to_f32 over all 65536 halves (stored as float32 bit patterns, compressed)
  quant.npz    jd_qmatvec and jd_dequant_any for every packed dtype on random blocks
  sample.npz   sample() on random logits for several temperatures / top-k / states
  own_depth4.npz   depth-4 own model, seed 0: 32-token prompt + 32 greedy tokens, EMA per
                   step, logits at three positions, md5 of export_gguf's file
  own_depth12.npz  depth-12 GQA 12/4 model with 5-8 alive experts per layer, seed 3: 10 steps
  host_q8.npz / host_q4k.npz  gguf_host_forward on synthetic GGUFs (written by the library's
                   generator, identified by md5) with a seeded LoRA parliament: 10 steps
  host_tokens.npz  host_tokenize and host_decode_print on a generated GGUF's vocabulary
Usage:  python tests/golden/gen_golden.py
"""
import ctypes as C
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

from oracle.oracle import Reference, fptr  # noqa: E402

OUT = HERE


def md5(path):
    return hashlib.md5(open(path, "rb").read()).hexdigest()


def rng_fixture(ref):
    L = ref.lib
    states = [1, 42, 0x9E3779B97F4A7C15, 123456789123]
    nxt, uni, nrm = [], [], []
    for s in states:
        L.jdr_rng_set(s)
        nxt.append([L.jdr_rng_next() for _ in range(64)])
        L.jdr_rng_set(s)
        uni.append([L.jdr_rand_uniform() for _ in range(64)])
        L.jdr_rng_set(s)
        nrm.append([L.jdr_rand_normal() for _ in range(64)])
    np.savez_compressed(os.path.join(OUT, "rng.npz"), states=np.array(states, np.uint64),
                        next=np.array(nxt, np.uint64), uniform=np.array(uni, np.float32),
                        normal=np.array(nrm, np.float32))


def f16_fixture(ref):
    out = np.array([ref.lib.jdr_f16_to_f32(h) for h in range(65536)], np.float32)
    np.savez_compressed(os.path.join(OUT, "f16.npz"), bits=out.view(np.uint32))


BLOCK = {1: (1, 2), 2: (32, 18), 6: (32, 22), 8: (32, 34), 12: (256, 144), 14: (256, 210)}


def random_packed(rng, dt, rows, cols):
    be, bb = BLOCK[dt]
    if dt == 1:
        h = (rng.standard_normal((rows, cols)) * 0.05).astype(np.float16)
        return h.view(np.uint8).reshape(rows, -1)
    nb = cols // be
    blk = rng.integers(0, 256, (rows, nb, bb)).astype(np.uint8)
    d = (rng.random((rows, nb)) * 1e-3 + 1e-4).astype(np.float16).view(np.uint8).reshape(rows, nb, 2)
    if dt == 14:
        blk[:, :, 208:210] = d
    else:
        blk[:, :, 0:2] = d
        if dt == 12:
            blk[:, :, 2:4] = (rng.random((rows, nb)) * 1e-3).astype(np.float16).view(np.uint8).reshape(rows, nb, 2)
    return blk.reshape(rows, -1)


def quant_fixture(ref):
    rng = np.random.default_rng(2024)
    d = {}
    for dt in sorted(BLOCK):
        rows, cols = 6, 512
        W = random_packed(rng, dt, rows, cols)
        x = rng.standard_normal(cols).astype(np.float32)
        y = ref.qmatvec(W, dt, x, rows, cols)
        dq = np.zeros(rows * cols, np.float32)
        assert ref.lib.jdr_dequant(W.ctypes.data_as(C.c_void_p), fptr(dq), rows * cols, dt) == 0
        d["W%d" % dt], d["x%d" % dt], d["y%d" % dt], d["dq%d" % dt] = W, x, y, dq
    np.savez_compressed(os.path.join(OUT, "quant.npz"), **d)


def sample_fixture(ref):
    rng = np.random.default_rng(77)
    cases = []
    for temp, topk in [(0.0, 0), (0.8, 40), (1.0, 0), (0.5, 5), (1.3, 100)]:
        for _ in range(6):
            lg = (rng.standard_normal(300) * 2).astype(np.float32)
            st = int(rng.integers(1, 2 ** 63))
            r, st2 = ref.sample(lg, temp, topk, st)
            cases.append((lg, temp, topk, st, r, st2))
    np.savez_compressed(os.path.join(OUT, "sample.npz"),
                        logits=np.array([c[0] for c in cases]), temp=np.array([c[1] for c in cases], np.float32),
                        topk=np.array([c[2] for c in cases], np.int32), state=np.array([c[3] for c in cases], np.uint64),
                        pick=np.array([c[4] for c in cases], np.int32), state_after=np.array([c[5] for c in cases], np.uint64))


def splitmix(x):
    m = (1 << 64) - 1
    z = (x + 0x9E3779B97F4A7C15) & m
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & m
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & m
    z = z ^ (z >> 31)
    return z or 1


def prompt(seq_seed, V, n):
    m = (1 << 64) - 1
    s = splitmix(seq_seed)
    out = []
    for _ in range(n):
        s ^= (s << 13) & m
        s ^= s >> 7
        s ^= (s << 17) & m
        s &= m
        out.append(s % V)
    return np.array(out, np.int32)


def own_fixture(ref, name, depth, kv, V, ctx, seed, masks, P, G, keep):
    ref.own_setup(depth, kv, V, ctx, seed, 0.02, masks)
    alive = np.array([ref.own_alive(l) for l in range(depth)], np.int32)
    path = "/tmp/jd_golden_%s.gguf" % name
    ref.lib.jdr_own_export(path.encode())
    h = md5(path)
    os.remove(path)
    ref.own_reset()
    toks = list(prompt(seed * 1000, V, P))
    emas, logits, lg = [], {}, None
    for pos in range(P + G - 1):
        lg, ema = ref.own_forward(toks[pos], pos)
        emas.append(ema)
        if pos in keep:
            logits[pos] = lg
        if pos + 1 >= P:
            toks.append(int(np.argmax(lg)))
    np.savez_compressed(os.path.join(OUT, "%s.npz" % name), tokens=np.array(toks, np.int32),
                        ema=np.array(emas, np.float32), alive=alive, gguf_md5=np.array(h),
                        logit_pos=np.array(sorted(logits), np.int32),
                        logits=np.array([logits[p] for p in sorted(logits)], np.float32),
                        cfg=np.array([depth, kv, V, ctx, seed, int(masks), P, G], np.int64))


HOST = {
    # name: arch, dim, layers, heads, kv, ffn, vocab, dtype, theta, rank, alive
    "host_q8": ("qwen2", 256, 2, 4, 2, 512, 1000, 8, 1e4, 8, 4),
    "host_q4k": ("llama", 512, 2, 4, 2, 1024, 2000, 12, 5e5, 16, 4),
}


def host_fixture(name):
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import conftest  # noqa: F401  (loads the package for the GGUF writer)
    import janus_doe_b200 as jd
    arch, D, L, H, KV, FF, V, dt, theta, R, na = HOST[name]
    path = "/tmp/jd_golden_%s.gguf" % name
    jd.write_synthetic_gguf(path, arch, L, D, FF, H, KV, V, theta, 1e-5, dt, 7, 0.02)
    ref = Reference("_r8" if R == 8 else "")
    ref.host_load(path)
    ref.lib.jdr_host_lora_seed(11, na, 0.01, 1.0 / D ** 0.5)
    ref.lib.jdr_host_reset_seq(64)
    toks = prompt(5, V, 10)
    lgs, emas = [], []
    for pos, t in enumerate(toks):
        lg, ema = ref.host_forward(int(t), pos)
        lgs.append(lg)
        emas.append(ema)
    ref.lib.jdr_host_free()
    np.savez_compressed(os.path.join(OUT, "%s.npz" % name), gguf_md5=np.array(md5(path)), tokens=toks,
                        logits=np.array(lgs, np.float32), ema=np.array(emas, np.float32))
    os.remove(path)


TOKEN_TEXTS = [b"", b"   ", b"a", b"zzqqy xylophone", "caf\u00e9 na\u00efve".encode(), b"k" * 150 + b" x",
               b"!@# $%^ &*()", b"<s> </s> <unk>", b"x" * 121, bytes(range(32, 127))]


def tokenizer_fixture():
    """host_tokenize / host_decode_print on the synthetic vocabulary of a generated GGUF:
    the texts above plus sentences of vocabulary words (every 7th word id from 98), and the
    printed form of ids -2..V+2."""
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import conftest  # noqa: F401
    import janus_doe_b200 as jd
    path = "/tmp/jd_golden_tok.gguf"
    V = 3000
    jd.write_synthetic_gguf(path, "llama", 1, 256, 512, 4, 2, V, 1e4, 1e-5, 8, 3, 0.02)
    ref = Reference("")
    ref.host_load(path)
    words = [ref.host_decode_print(i).strip() for i in range(98, V, 7)]
    texts = TOKEN_TEXTS + [b" ".join(words[i:i + 40]) for i in range(0, len(words), 40)]
    ids, lens = [], []
    for t in texts:
        r = ref.host_tokenize(t, 256)
        ids += r
        lens.append(len(r))
    printed = [ref.host_decode_print(i) for i in range(-2, V + 3)]
    ref.lib.jdr_host_free()
    np.savez_compressed(os.path.join(OUT, "host_tokens.npz"), gguf_md5=np.array(md5(path)),
                        texts=np.array(texts, dtype=object), ids=np.array(ids, np.int32), lens=np.array(lens, np.int32),
                        printed=np.array(printed, dtype=object))
    os.remove(path)


def main():
    ref = Reference("")
    rng_fixture(ref)
    f16_fixture(ref)
    quant_fixture(ref)
    sample_fixture(ref)
    own_fixture(ref, "own_depth4", 4, 0, 2256, 256, 0, False, 32, 32, {0, 31, 62})
    own_fixture(ref, "own_depth12", 12, 4, 8256, 1024, 3, True, 6, 4, {8})
    for name in HOST:
        host_fixture(name)
    tokenizer_fixture()
    print("fixtures written to", OUT)


if __name__ == "__main__":
    main()
