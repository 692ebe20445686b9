"""ctypes bindings to the parity oracle (TEST INFRASTRUCTURE ONLY).

`Oracle` wraps libjdoracle.so, the C restatement of the reference decode path
(jd_oracle.c).  `Reference` wraps oracle/_ref/libjdref*.so, the reference's own
source compiled by oracle/Makefile through ref_harness.c.  Only tests, the smoke
check and bench.py's CPU-baseline leg import this module; the product never does.
"""
import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
MAXE = 16
MAXL = 32
F32P = C.POINTER(C.c_float)
I32P = C.POINTER(C.c_int)


def fptr(a):
    return a.ctypes.data_as(F32P)


def iptr(a):
    return a.ctypes.data_as(I32P)


class JdoConfig(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("depth", "dim", "n_heads", "n_kv_heads", "head_dim",
                                        "hidden_dim", "vocab_size", "seq_len")] + \
               [("norm_eps", C.c_float), ("rope_theta", C.c_float), ("attn_clamp", C.c_float),
                ("active_depth", C.c_int), ("initial_experts", C.c_int)]


class JdoLayer(C.Structure):
    _fields_ = [(n, F32P) for n in ("attn_norm", "ffn_norm", "wq", "wk", "wv", "wo", "w_vote")] + \
               [("w_gate", F32P * MAXE), ("w_up", F32P * MAXE), ("w_down", F32P * MAXE),
                ("alive", C.c_int * MAXE), ("consensus", C.c_float), ("temperature", C.c_float)]


class JdoOwn(C.Structure):
    _fields_ = [("c", JdoConfig), ("tok_emb", F32P), ("output", F32P), ("output_norm", F32P),
                ("layers", JdoLayer * MAXL)]


class JdoOwnState(C.Structure):
    _fields_ = [(n, F32P) for n in ("key_cache", "value_cache", "cos_cache", "sin_cache")] + \
               [("consensus", C.c_float * MAXL)] + \
               [(n, F32P) for n in ("x", "xb", "xb2", "hb", "hb2", "q", "k", "v", "att", "logits", "expert_out")]


class JdoElect(C.Structure):
    _fields_ = [("k", C.c_int), ("n_alive", C.c_int), ("sel", C.c_int * MAXE), ("w", C.c_float * MAXE),
                ("votes", C.c_float * MAXE), ("ema", C.c_float)]


class _HostLayer(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("wq", "wk", "wv", "wo", "gate", "up", "down")] + \
               [(n, C.c_int) for n in ("wq_dt", "wk_dt", "wv_dt", "wo_dt", "gate_dt", "up_dt", "down_dt")] + \
               [("attn_norm", F32P), ("ffn_norm", F32P)]


class JdoHost(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("n_layers", "dim", "hidden", "n_heads", "n_kv_heads", "head_dim", "vocab")] + \
               [("rope_theta", C.c_float), ("rms_eps", C.c_float), ("rope_norm", C.c_int), ("arch", C.c_char * 64),
                ("bos", C.c_int), ("eos", C.c_int), ("map", C.c_void_p), ("map_size", C.c_size_t),
                ("tok_emb", F32P), ("output", C.c_void_p), ("output_dt", C.c_int), ("output_norm", F32P),
                ("layers", _HostLayer * MAXL), ("dq", F32P * (MAXL * 3 + 4)), ("n_dq", C.c_int),
                ("lora_rank", C.c_int), ("lora_alpha", C.c_float), ("w_vote", F32P * MAXL),
                ("A", (F32P * MAXE) * MAXL), ("B", (F32P * MAXE) * MAXL), ("alive", (C.c_int * MAXE) * MAXL),
                ("consensus0", C.c_float * MAXL), ("attention_bias", C.c_float * MAXL),
                ("layer_focus", C.c_float * MAXL)]


class JdoHostState(C.Structure):
    _fields_ = [("max_seq", C.c_int), ("kc", F32P), ("vc", F32P), ("consensus", C.c_float * MAXL),
                ("host_x", F32P), ("host_dy", F32P), ("tokens_seen", (C.c_int * MAXE) * MAXL)]


def trace_to_arrays(tr, L):
    """Turn a JdoElect[L] into dict of numpy arrays (k, sel, w, ema, n_alive)."""
    k = np.array([tr[l].k for l in range(L)], np.int32)
    sel = np.full((L, MAXE), -1, np.int32)
    w = np.zeros((L, MAXE), np.float32)
    for l in range(L):
        for i in range(tr[l].k):
            sel[l, i] = tr[l].sel[i]
            w[l, i] = tr[l].w[i]
    ema = np.array([tr[l].ema for l in range(L)], np.float32)
    votes = np.array([[tr[l].votes[e] for e in range(MAXE)] for l in range(L)], np.float32)
    n_alive = np.array([tr[l].n_alive for l in range(L)], np.int32)
    return {"k": k, "sel": sel, "w": w, "ema": ema, "votes": votes, "n_alive": n_alive}


class Oracle:
    """The C restatement (jd_oracle.c)."""

    def __init__(self, path=None):
        path = path or os.path.join(HERE, "libjdoracle.so")
        if not os.path.exists(path):
            raise RuntimeError("oracle not built: run `make -C oracle`")
        L = self.lib = C.CDLL(path)
        L.jdo_splitmix64.restype = C.c_uint64
        L.jdo_splitmix64.argtypes = [C.c_uint64]
        L.jdo_rng_next.restype = C.c_uint64
        L.jdo_rng_next.argtypes = [C.POINTER(C.c_uint64)]
        L.jdo_rand_uniform.restype = C.c_float
        L.jdo_rand_uniform.argtypes = [C.POINTER(C.c_uint64)]
        L.jdo_rand_normal.restype = C.c_float
        L.jdo_rand_normal.argtypes = [C.POINTER(C.c_uint64)]
        L.jdo_config_from_depth.argtypes = [C.c_int, C.POINTER(JdoConfig)]
        L.jdo_own_alloc.argtypes = [C.POINTER(JdoOwn), C.POINTER(JdoConfig)]
        L.jdo_own_fill_seeded.argtypes = [C.POINTER(JdoOwn), C.c_uint64, C.c_float, C.c_int]
        L.jdo_own_free.argtypes = [C.POINTER(JdoOwn)]
        L.jdo_own_state_alloc.argtypes = [C.POINTER(JdoOwn), C.POINTER(JdoOwnState)]
        L.jdo_own_state_reset.argtypes = [C.POINTER(JdoOwn), C.POINTER(JdoOwnState)]
        L.jdo_own_state_free.argtypes = [C.POINTER(JdoOwnState)]
        L.jdo_own_forward.restype = F32P
        L.jdo_own_forward.argtypes = [C.POINTER(JdoOwn), C.POINTER(JdoOwnState), C.c_int, C.c_int, C.POINTER(JdoElect)]
        L.jdo_sample.argtypes = [F32P, C.c_int, C.c_float, C.c_int, C.POINTER(C.c_uint64)]
        L.jdo_argmax.argtypes = [F32P, C.c_int]
        L.jdo_prompt.argtypes = [C.c_uint64, C.c_int, C.c_int, I32P, C.POINTER(C.c_uint64)]
        L.jdo_f16_to_f32.restype = C.c_float
        L.jdo_f16_to_f32.argtypes = [C.c_uint16]
        L.jdo_dequant.argtypes = [C.c_void_p, F32P, C.c_uint64, C.c_int]
        L.jdo_qmatvec.argtypes = [F32P, C.c_void_p, C.c_int, F32P, C.c_int, C.c_int]
        L.jdo_matvec.argtypes = [F32P, F32P, F32P, C.c_int, C.c_int]
        L.jdo_set_threads.argtypes = [C.c_int]
        L.jdo_host_load.argtypes = [C.POINTER(JdoHost), C.c_char_p, C.c_int, C.c_int]
        L.jdo_host_lora_seed.argtypes = [C.POINTER(JdoHost), C.c_uint64, C.c_int, C.c_float, C.c_float]
        L.jdo_host_free.argtypes = [C.POINTER(JdoHost)]
        L.jdo_host_state_alloc.argtypes = [C.POINTER(JdoHost), C.POINTER(JdoHostState), C.c_int]
        L.jdo_host_state_reset.argtypes = [C.POINTER(JdoHost), C.POINTER(JdoHostState)]
        L.jdo_host_state_free.argtypes = [C.POINTER(JdoHostState)]
        L.jdo_host_forward.argtypes = [C.POINTER(JdoHost), C.POINTER(JdoHostState), C.c_int, C.c_int, F32P,
                                       C.POINTER(JdoElect)]
        L.jdo_host_elect.argtypes = [C.POINTER(JdoHost), C.c_int, C.POINTER(C.c_float), F32P, C.c_int, I32P, F32P,
                                     C.POINTER(JdoElect)]
        L.jdo_host_learn_run.argtypes = [C.POINTER(JdoHost), C.POINTER(JdoHostState), I32P, C.c_int, C.c_float,
                                         C.POINTER(C.c_uint64), I32P]

    # ---- helpers
    def splitmix64(self, x):
        return self.lib.jdo_splitmix64(x)

    def config(self, depth, **over):
        c = JdoConfig()
        self.lib.jdo_config_from_depth(depth, C.byref(c))
        for k, v in over.items():
            setattr(c, k, v)
        return c

    def prompt(self, seq_seed, V, n):
        out = np.zeros(n, np.int32)
        st = C.c_uint64(0)
        self.lib.jdo_prompt(seq_seed, V, n, iptr(out), C.byref(st))
        return out, st.value

    def sample(self, logits, temp, top_k, state):
        lg = np.array(logits, np.float32, copy=True)
        st = C.c_uint64(state)
        r = self.lib.jdo_sample(fptr(lg), lg.size, temp, top_k, C.byref(st))
        return r, st.value

    def qmatvec(self, W, dt, x, r, c):
        out = np.zeros(r, np.float32)
        x = np.ascontiguousarray(x, np.float32)
        rc = self.lib.jdo_qmatvec(fptr(out), W.ctypes.data_as(C.c_void_p), dt, fptr(x), r, c)
        if rc != 0:
            raise ValueError("unsupported dtype/shape")
        return out

    def dequant(self, W, n, dt):
        out = np.zeros(n, np.float32)
        if self.lib.jdo_dequant(W.ctypes.data_as(C.c_void_p), fptr(out), n, dt) != 0:
            raise ValueError("unsupported dtype")
        return out


class OwnModel:
    """Seeded own model + per-sequence decode on the oracle."""

    def __init__(self, orc, cfg, seed, std=0.02, draw_masks=False):
        self.orc, self.lib = orc, orc.lib
        self.m = JdoOwn()
        if self.lib.jdo_own_alloc(C.byref(self.m), C.byref(cfg)) != 0:
            raise MemoryError("oracle alloc failed")
        self.lib.jdo_own_fill_seeded(C.byref(self.m), seed, std, 1 if draw_masks else 0)
        self.c = self.m.c
        self.s = JdoOwnState()
        self.lib.jdo_own_state_alloc(C.byref(self.m), C.byref(self.s))
        self.tr = (JdoElect * MAXL)()

    def alive(self, l):
        return [self.m.layers[l].alive[e] for e in range(MAXE)]

    def reset(self):
        self.lib.jdo_own_state_reset(C.byref(self.m), C.byref(self.s))

    def forward(self, tok, pos, trace=False):
        p = self.lib.jdo_own_forward(C.byref(self.m), C.byref(self.s), int(tok), int(pos),
                                     self.tr if trace else None)
        lg = np.ctypeslib.as_array(p, shape=(self.c.vocab_size,)).copy()
        if trace:
            return lg, trace_to_arrays(self.tr, self.c.active_depth or self.c.depth)
        return lg

    def ema(self):
        return np.array(self.s.consensus[: self.c.depth], np.float32)

    def close(self):
        if self.m.tok_emb:
            self.lib.jdo_own_state_free(C.byref(self.s))
            self.lib.jdo_own_free(C.byref(self.m))


class OwnSeq:
    """One more decode state (KV, per-layer EMA, scratch) over an OwnModel's weights, so that
    several sequences can run on the oracle at once (one state per thread; the ctypes call
    releases the GIL and the forward touches only its own state)."""

    def __init__(self, om):
        self.om, self.lib, self.c = om, om.lib, om.c
        self.s = JdoOwnState()
        if self.lib.jdo_own_state_alloc(C.byref(om.m), C.byref(self.s)) != 0:
            raise MemoryError("oracle state alloc failed")
        self.tr = (JdoElect * MAXL)()

    def reset(self):
        self.lib.jdo_own_state_reset(C.byref(self.om.m), C.byref(self.s))

    def forward(self, tok, pos, trace=False):
        p = self.lib.jdo_own_forward(C.byref(self.om.m), C.byref(self.s), int(tok), int(pos),
                                     self.tr if trace else None)
        lg = np.ctypeslib.as_array(p, shape=(self.c.vocab_size,)).copy()
        if trace:
            return lg, trace_to_arrays(self.tr, self.c.active_depth or self.c.depth)
        return lg

    def close(self):
        if self.s.x:
            self.lib.jdo_own_state_free(C.byref(self.s))


class HostModel:
    """Host GGUF model on the oracle."""

    def __init__(self, orc, path, lora_rank, rope_override=-1, max_seq=256):
        self.orc, self.lib = orc, orc.lib
        self.h = JdoHost()
        if not self.lib.jdo_host_load(C.byref(self.h), path.encode(), rope_override, lora_rank):
            raise ValueError("oracle: GGUF load failed: %s" % path)
        self.s = JdoHostState()
        self.max_seq = max_seq
        self.lib.jdo_host_state_alloc(C.byref(self.h), C.byref(self.s), max_seq)
        self.tr = (JdoElect * MAXL)()

    def lora_seed(self, seed, n_alive, ab_std, vote_amp):
        self.lib.jdo_host_lora_seed(C.byref(self.h), seed, n_alive, ab_std, vote_amp)

    def reset(self):
        self.lib.jdo_host_state_reset(C.byref(self.h), C.byref(self.s))

    def forward(self, tok, pos, trace=False):
        lg = np.zeros(self.h.vocab, np.float32)
        self.lib.jdo_host_forward(C.byref(self.h), C.byref(self.s), int(tok), int(pos), fptr(lg),
                                  self.tr if trace else None)
        if trace:
            return lg, trace_to_arrays(self.tr, self.h.n_layers)
        return lg

    def ema(self):
        return np.array(self.s.consensus[: self.h.n_layers], np.float32)

    def learn(self, toks, lr, rng, offset):
        """host_learn_run over toks; returns (deaths, rng, offset)."""
        t = np.ascontiguousarray(toks, np.int32)
        st, off = C.c_uint64(rng), C.c_int(offset)
        d = self.lib.jdo_host_learn_run(C.byref(self.h), C.byref(self.s), iptr(t), t.size, lr, C.byref(st),
                                        C.byref(off))
        return d, st.value, off.value

    def expert(self, l, e):
        """(A [D][R], B [R][D], alive) of expert slot e in layer l."""
        D, R = self.h.dim, self.h.lora_rank
        A = np.ctypeslib.as_array(self.h.A[l][e], (D, R)).copy() if self.h.A[l][e] else None
        B = np.ctypeslib.as_array(self.h.B[l][e], (R, D)).copy() if self.h.B[l][e] else None
        return A, B, int(self.h.alive[l][e])

    def close(self):
        if self.h.map:
            self.lib.jdo_host_state_free(C.byref(self.s))
            self.lib.jdo_host_free(C.byref(self.h))


class Reference:
    """The reference's own code (oracle/_ref/libjdref*.so, built by `make -C oracle ref`)."""

    def __init__(self, variant=""):
        path = os.path.join(HERE, "_ref", "libjdref%s.so" % variant)
        if not os.path.exists(path):
            raise RuntimeError("reference harness not built: %s" % path)
        L = self.lib = C.CDLL(path)
        L.jdr_rng_set.argtypes = [C.c_uint64]
        L.jdr_rng_get.restype = C.c_uint64
        L.jdr_rng_next.restype = C.c_uint64
        L.jdr_rand_uniform.restype = C.c_float
        L.jdr_rand_normal.restype = C.c_float
        L.jdr_own_setup.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_uint64, C.c_float, C.c_int]
        L.jdr_own_dims.argtypes = [I32P]
        L.jdr_own_alive.argtypes = [C.c_int, I32P]
        L.jdr_own_tensor.argtypes = [C.c_int, C.c_int, C.c_int, F32P, C.c_long]
        L.jdr_own_forward.argtypes = [C.c_int, C.c_int, F32P, F32P]
        L.jdr_own_export.argtypes = [C.c_char_p]
        L.jdr_own_load.argtypes = [C.c_char_p]
        L.jdr_sample.argtypes = [F32P, C.c_int, C.c_float, C.c_int, C.POINTER(C.c_uint64)]
        L.jdr_f16_to_f32.restype = C.c_float
        L.jdr_f16_to_f32.argtypes = [C.c_uint16]
        L.jdr_dequant.argtypes = [C.c_void_p, F32P, C.c_uint64, C.c_int]
        L.jdr_qmatvec.argtypes = [F32P, C.c_void_p, C.c_int, F32P, C.c_int, C.c_int]
        L.jdr_host_load.argtypes = [C.c_char_p, C.c_int]
        L.jdr_host_dims.argtypes = [I32P]
        L.jdr_host_theta.restype = C.c_float
        L.jdr_host_eps.restype = C.c_float
        L.jdr_host_lora_seed.argtypes = [C.c_uint64, C.c_int, C.c_float, C.c_float]
        L.jdr_host_reset_seq.argtypes = [C.c_int]
        L.jdr_host_forward.argtypes = [C.c_int, C.c_int, F32P, F32P]
        L.jdr_host_tokenize.argtypes = [C.c_char_p, I32P, C.c_int]
        L.jdr_host_learn.argtypes = [I32P, C.c_int, C.c_int, C.c_float, C.POINTER(C.c_uint64), I32P]
        L.jdr_host_expert.argtypes = [C.c_int, C.c_int, F32P, F32P]
        L.jdr_host_decode_print.argtypes = [C.c_int, C.c_char_p, C.c_int]
        self.depth = 0
        self.V = 0

    def own_setup(self, depth, n_kv, vocab, seq_len, seed, std=0.02, draw_masks=False):
        self.lib.jdr_own_setup(depth, n_kv, vocab, seq_len, seed, std, 1 if draw_masks else 0)
        d = np.zeros(9, np.int32)
        self.lib.jdr_own_dims(iptr(d))
        self.dims = d
        self.depth, self.V = int(d[0]), int(d[6])

    def own_alive(self, l):
        a = np.zeros(MAXE, np.int32)
        self.lib.jdr_own_alive(l, iptr(a))
        return list(a)

    def own_forward(self, tok, pos):
        lg = np.zeros(self.V, np.float32)
        ema = np.zeros(self.depth, np.float32)
        self.lib.jdr_own_forward(int(tok), int(pos), fptr(lg), fptr(ema))
        return lg, ema

    def own_reset(self):
        self.lib.jdr_own_reset_seq()

    def sample(self, logits, temp, top_k, state):
        lg = np.array(logits, np.float32, copy=True)
        st = C.c_uint64(state)
        r = self.lib.jdr_sample(fptr(lg), lg.size, temp, top_k, C.byref(st))
        return r, st.value

    def qmatvec(self, W, dt, x, r, c):
        out = np.zeros(r, np.float32)
        x = np.ascontiguousarray(x, np.float32)
        if self.lib.jdr_qmatvec(fptr(out), W.ctypes.data_as(C.c_void_p), dt, fptr(x), r, c) != 0:
            raise ValueError("unsupported")
        return out

    def host_load(self, path, rope_override=-1):
        if not self.lib.jdr_host_load(path.encode(), rope_override):
            raise ValueError("reference: GGUF load failed")
        d = np.zeros(11, np.int32)
        self.lib.jdr_host_dims(iptr(d))
        self.hdims = d
        self.hL, self.hV = int(d[0]), int(d[6])

    def host_learn(self, toks, max_seq, lr, rng, offset):
        t = np.ascontiguousarray(toks, np.int32)
        st, off = C.c_uint64(rng), C.c_int(offset)
        d = self.lib.jdr_host_learn(iptr(t), t.size, max_seq, lr, C.byref(st), C.byref(off))
        return d, st.value, off.value

    def host_expert(self, l, e):
        D, R = int(self.hdims[1]), int(self.lib.jdr_lora_rank())
        A = np.zeros((D, R), np.float32)
        B = np.zeros((R, D), np.float32)
        alive = self.lib.jdr_host_expert(l, e, fptr(A), fptr(B))
        return A, B, int(alive)

    def host_tokenize(self, text, max_ids=256):
        out = np.zeros(max(1, max_ids), np.int32)
        n = self.lib.jdr_host_tokenize(text if isinstance(text, bytes) else text.encode(), iptr(out), max_ids)
        return [int(t) for t in out[:n]]

    def host_decode_print(self, tok):
        buf = C.create_string_buffer(512)
        n = self.lib.jdr_host_decode_print(int(tok), buf, 512)
        return buf.raw[:max(0, n)]

    def host_forward(self, tok, pos):
        lg = np.zeros(self.hV, np.float32)
        ema = np.zeros(self.hL, np.float32)
        self.lib.jdr_host_forward(int(tok), int(pos), fptr(lg), fptr(ema))
        return lg, ema
