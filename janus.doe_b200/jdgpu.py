"""Python binding of the B200 decode engine: ctypes over the C ABI in include/jdgpu.h.

The engine is libjdgpu.so in this directory (built by build.py).  There is no CPU or
PyTorch fallback: importing this module on a machine without the built library, or
opening a context without a B200, raises.
"""
import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libjdgpu.so")
MAXE = 16
MAXL = 32
F32P = C.POINTER(C.c_float)
I32P = C.POINTER(C.c_int)
U64P = C.POINTER(C.c_uint64)

JD_OK, JD_EINVAL, JD_ENOMEM, JD_ECUDA, JD_EFORMAT, JD_EUNSUPPORTED, JD_EIO, JD_ESTATE, JD_ECOMM = 0, -1, -2, -3, -4, -5, -6, -7, -8
JD_F32, JD_F16, JD_Q4_0, JD_Q5_0, JD_Q8_0, JD_Q4_K, JD_Q6_K = 0, 1, 2, 6, 8, 12, 14
STATUS = {0: "ok", -1: "invalid argument", -2: "out of memory", -3: "CUDA error", -4: "bad format",
          -5: "unsupported", -6: "I/O error", -7: "bad state", -8: "NCCL error"}


class JdError(RuntimeError):
    def __init__(self, code, msg=""):
        super().__init__("%s (%d)%s" % (STATUS.get(code, "error"), code, (": " + msg) if msg else ""))
        self.code = code


class JdConfig(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("depth", "dim", "n_heads", "n_kv_heads", "head_dim", "hidden_dim",
                                        "vocab_size", "seq_len")] + \
               [("norm_eps", C.c_float), ("rope_theta", C.c_float), ("attn_clamp", C.c_float),
                ("active_depth", C.c_int), ("initial_experts", C.c_int)]


class JdLayer(C.Structure):
    _fields_ = [(n, F32P) for n in ("attn_norm", "ffn_norm", "wq", "wk", "wv", "wo", "w_vote")] + \
               [("w_gate", F32P * MAXE), ("w_up", F32P * MAXE), ("w_down", F32P * MAXE),
                ("alive", C.c_int * MAXE), ("consensus", C.c_float), ("temperature", C.c_float)]


class JdModel(C.Structure):
    _fields_ = [("c", JdConfig), ("tok_emb", F32P), ("output", F32P), ("output_norm", F32P),
                ("layers", JdLayer * MAXL)]


class JdHostLayer(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("wq", "wk", "wv", "wo", "gate", "up", "down")] + \
               [(n, C.c_int) for n in ("wq_dt", "wk_dt", "wv_dt", "wo_dt", "gate_dt", "up_dt", "down_dt")] + \
               [("attn_norm", F32P), ("ffn_norm", F32P)]


class JdHostModel(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("n_layers", "dim", "hidden", "n_heads", "n_kv_heads", "head_dim", "vocab")] + \
               [("rope_theta", C.c_float), ("rms_eps", C.c_float), ("rope_norm", C.c_int), ("arch", C.c_char * 64),
                ("bos", C.c_int), ("eos", C.c_int), ("tok_emb", F32P), ("output", C.c_void_p), ("output_dt", C.c_int),
                ("output_norm", F32P), ("layers", JdHostLayer * MAXL), ("lora_rank", C.c_int),
                ("lora_alpha", C.c_float), ("w_vote", F32P * MAXL), ("A", (F32P * MAXE) * MAXL),
                ("B", (F32P * MAXE) * MAXL), ("alive", (C.c_int * MAXE) * MAXL), ("consensus0", C.c_float * MAXL),
                ("attention_bias", C.c_float * MAXL), ("layer_focus", C.c_float * MAXL),
                ("vocab_tokens", C.POINTER(C.c_char_p)), ("n_vocab_tokens", C.c_int), ("priv", C.c_void_p)]


class JdTpShard(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("q_head0", "q_heads", "kv_head0", "kv_heads", "hidden0", "hidden",
                                        "vocab0", "vocab")]


class JdgTrace(C.Structure):
    _fields_ = [("k", I32P), ("sel", I32P), ("w", F32P), ("ema", F32P)]


_lib = None


def lib():
    """Load libjdgpu.so (fails loudly when it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError("libjdgpu.so is not built; run `python janus.doe_b200/build.py`")
    L = C.CDLL(LIB_PATH)
    sig = {
        "jd_config_from_depth": [C.c_int, C.POINTER(JdConfig)],
        "jd_model_alloc": [C.POINTER(JdModel), C.POINTER(JdConfig)],
        "jd_model_free": [C.POINTER(JdModel)],
        "jd_model_fill_seeded": [C.POINTER(JdModel), C.c_uint64, C.c_float, C.c_int],
        "jd_model_export_gguf": [C.POINTER(JdModel), C.c_char_p],
        "jd_model_load_gguf": [C.POINTER(JdModel), C.c_char_p],
        "jd_host_load_gguf": [C.POINTER(JdHostModel), C.c_char_p, C.c_int, C.c_int],
        "jd_host_free": [C.POINTER(JdHostModel)],
        "jd_host_lora_seed": [C.POINTER(JdHostModel), C.c_uint64, C.c_int, C.c_float, C.c_float],
        "jd_host_lora_save": [C.POINTER(JdHostModel), C.c_char_p],
        "jd_host_lora_load": [C.POINTER(JdHostModel), C.c_char_p],
        "jd_gguf_write_synthetic": [C.c_char_p, C.c_char_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                    C.c_float, C.c_float, C.c_int, C.c_uint64, C.c_float, C.c_int],
        "jd_gguf_write_synthetic_mixed": [C.c_char_p, C.c_char_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                          C.c_int, C.c_float, C.c_float, C.c_int, C.c_int, C.c_uint64, C.c_float,
                                          C.c_int],
        "jd_dequant": [C.c_void_p, F32P, C.c_uint64, C.c_int],
        "jd_tp_shard_of": [C.POINTER(JdHostModel), C.c_int, C.c_int, C.c_void_p],
        "jd_host_tokenize": [C.POINTER(JdHostModel), C.c_char_p, I32P, C.c_int],
        "jd_host_token_text": [C.POINTER(JdHostModel), C.c_int, C.c_char_p, C.c_int],
        "jdg_open": [C.c_int, C.POINTER(C.c_void_p)],
        "jdg_close": [C.c_void_p],
        "jdg_last_error": [C.c_void_p],
        "jdg_device_count": [I32P],
        "jdg_own_upload": [C.c_void_p, C.POINTER(JdModel), C.c_int, C.POINTER(C.c_void_p)],
        "jdg_host_upload": [C.c_void_p, C.POINTER(JdHostModel), C.c_int, C.c_int, C.POINTER(C.c_void_p)],
        "jdg_comm_unique_id": [C.c_void_p],
        "jdg_host_upload_tp": [C.c_void_p, C.POINTER(JdHostModel), C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p,
                               C.POINTER(C.c_void_p)],
        "jdg_engine_free": [C.c_void_p],
        "jdg_set_sampling": [C.c_void_p, C.c_float, C.c_int],
        "jdg_reset": [C.c_void_p, C.c_int],
        "jdg_set_prompt": [C.c_void_p, C.c_int, I32P, C.c_int, I32P, U64P],
        "jdg_run": [C.c_void_p, C.c_int, C.c_int],
        "jdg_prefill": [C.c_void_p, C.c_int],
        "jdg_host_learn": [C.c_void_p, I32P, C.c_int, C.c_float, U64P, I32P, I32P],
        "jdg_host_get_expert": [C.c_void_p, C.c_int, C.c_int, F32P, F32P, I32P],
        "jdg_get_prefill_trace": [C.c_void_p, C.c_int, C.POINTER(JdgTrace)],
        "jdg_get_state": [C.c_void_p, C.c_int, I32P, I32P],
        "jdg_get_history": [C.c_void_p, C.c_int, C.c_int, I32P],
        "jdg_step": [C.c_void_p, C.c_int, I32P, I32P, U64P, I32P, F32P, C.POINTER(JdgTrace)],
        "jdg_get_logits": [C.c_void_p, C.c_int, F32P],
        "jdg_get_trace": [C.c_void_p, C.c_int, C.POINTER(JdgTrace)],
        "jdg_last_run_ms": [C.c_void_p, F32P],
        "jdg_launch_count": [C.c_void_p, C.POINTER(C.c_longlong)],
        "jdg_get_stats": [C.c_void_p, U64P],
        "jdg_reset_stats": [C.c_void_p],
        "jdg_debug_timeline": [C.c_void_p, C.c_int, U64P],
        "jdg_qmatvec": [C.c_void_p, F32P, C.c_void_p, C.c_int, F32P, C.c_int, C.c_int, C.c_int],
    }
    for name, args in sig.items():
        f = getattr(L, name)
        f.argtypes = args
        f.restype = C.c_int
    L.jd_model_free.restype = None
    L.jd_host_free.restype = None
    L.jdg_close.restype = None
    L.jdg_engine_free.restype = None
    L.jdg_last_error.restype = C.c_char_p
    _lib = L
    return L


def exported_symbols():
    """Names of the jd_/jdg_ entry points the header declares (for ABI checks)."""
    import re
    hdr = open(os.path.join(os.path.dirname(HERE), "include", "jdgpu.h")).read()
    return sorted(set(re.findall(r"\b(jdg?_[a-z0-9_]+)\s*\(", hdr)) - {"jd_config", "jd_model"})


def _p(a, t):
    return a.ctypes.data_as(t)


def check(rc, ctx=None):
    if rc != JD_OK:
        msg = lib().jdg_last_error(ctx)
        raise JdError(rc, msg.decode(errors="replace") if msg else "")
    return rc


# --------------------------------------------------------------------------- host model code
def config_from_depth(depth, **over):
    c = JdConfig()
    check(lib().jd_config_from_depth(depth, C.byref(c)))
    for k, v in over.items():
        setattr(c, k, v)
    return c


class Model:
    """The own model on the host (jd_model): allocate, seed, export/load GGUF."""

    def __init__(self, cfg):
        self.m = JdModel()
        check(lib().jd_model_alloc(C.byref(self.m), C.byref(cfg)))

    @classmethod
    def seeded(cls, cfg, seed, std=0.02, draw_masks=False):
        m = cls(cfg)
        check(lib().jd_model_fill_seeded(C.byref(m.m), seed, std, 1 if draw_masks else 0))
        return m

    @property
    def c(self):
        return self.m.c

    def alive(self, l):
        return [self.m.layers[l].alive[e] for e in range(MAXE)]

    def export_gguf(self, path):
        check(lib().jd_model_export_gguf(C.byref(self.m), path.encode()))

    def load_gguf(self, path):
        check(lib().jd_model_load_gguf(C.byref(self.m), path.encode()))

    def close(self):
        if self.m.tok_emb:
            lib().jd_model_free(C.byref(self.m))

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class HostModel:
    """A host GGUF model on the host (jd_host_model)."""

    def __init__(self, path, lora_rank=16, rope_override=-1):
        self.h = JdHostModel()
        check(lib().jd_host_load_gguf(C.byref(self.h), path.encode(), rope_override, lora_rank))

    def lora_seed(self, seed, n_alive, ab_std, vote_amp):
        check(lib().jd_host_lora_seed(C.byref(self.h), seed, n_alive, ab_std, vote_amp))

    def lora_save(self, path):
        check(lib().jd_host_lora_save(C.byref(self.h), path.encode()))

    def lora_load(self, path):
        check(lib().jd_host_lora_load(C.byref(self.h), path.encode()))

    def tokenize(self, text, max_ids=256):
        """host_tokenize: ids of the words of text (bytes or str)."""
        out = np.zeros(max(1, max_ids), np.int32)
        n = lib().jd_host_tokenize(C.byref(self.h), text if isinstance(text, bytes) else text.encode(),
                                   _p(out, I32P), max_ids)
        check(min(n, 0))
        return [int(t) for t in out[:n]]

    def token_text(self, tok):
        """The printable form of token tok (bytes)."""
        buf = C.create_string_buffer(512)
        n = lib().jd_host_token_text(C.byref(self.h), int(tok), buf, 512)
        check(min(n, 0))
        return buf.raw[:n]

    def close(self):
        if self.h.priv:
            lib().jd_host_free(C.byref(self.h))

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def write_synthetic_gguf(path, arch, n_layers, dim, hidden, n_heads, n_kv_heads, vocab, rope_theta, rms_eps, dtype,
                         seed, std=0.02, threads=0, out_dtype=None):
    if out_dtype is None:
        check(lib().jd_gguf_write_synthetic(path.encode(), arch.encode(), n_layers, dim, hidden, n_heads, n_kv_heads,
                                            vocab, rope_theta, rms_eps, dtype, seed, std, threads))
    else:
        check(lib().jd_gguf_write_synthetic_mixed(path.encode(), arch.encode(), n_layers, dim, hidden, n_heads,
                                                  n_kv_heads, vocab, rope_theta, rms_eps, dtype, out_dtype, seed, std,
                                                  threads))


def dequant(W, n, dt):
    """n weights of GGUF type dt (packed bytes W) decoded to f32 on the host."""
    W = np.ascontiguousarray(W)
    out = np.zeros(n, np.float32)
    check(lib().jd_dequant(W.ctypes.data_as(C.c_void_p), _p(out, F32P), n, dt))
    return out


# --------------------------------------------------------------------------- GPU engine
def device_count():
    n = C.c_int(0)
    lib().jdg_device_count(C.byref(n))
    return n.value


class Context:
    def __init__(self, device=0):
        self.h = C.c_void_p()
        rc = lib().jdg_open(device, C.byref(self.h))
        if rc != JD_OK:
            raise JdError(rc, (lib().jdg_last_error(None) or b"").decode())

    def check(self, rc):
        return check(rc, self.h)

    def close(self):
        if self.h:
            lib().jdg_close(self.h)
            self.h = C.c_void_p()


class Engine:
    """Uploaded model + per-sequence state on one GPU."""

    def __init__(self, ctx, handle, n_layers, vocab, ldl=None):
        # ldl: logits per sequence held by this engine (the rank's vocabulary slice under
        # tensor parallelism, the whole vocabulary otherwise)
        self.ctx, self.h, self.L, self.V = ctx, handle, n_layers, vocab
        self.ldl = vocab if ldl is None else ldl

    @classmethod
    def own(cls, ctx, model, max_batch=1):
        h = C.c_void_p()
        ctx.check(lib().jdg_own_upload(ctx.h, C.byref(model.m), max_batch, C.byref(h)))
        c = model.c
        L = c.active_depth if 0 < c.active_depth <= c.depth else c.depth
        return cls(ctx, h, L, c.vocab_size)

    @classmethod
    def host(cls, ctx, hm, max_batch=1, max_seq=256):
        h = C.c_void_p()
        ctx.check(lib().jdg_host_upload(ctx.h, C.byref(hm.h), max_batch, max_seq, C.byref(h)))
        return cls(ctx, h, min(hm.h.n_layers, MAXL), hm.h.vocab)

    @classmethod
    def host_tp(cls, ctx, hm, max_batch, max_seq, rank, world, nccl_id):
        h = C.c_void_p()
        buf = C.create_string_buffer(bytes(nccl_id), 128)
        ctx.check(lib().jdg_host_upload_tp(ctx.h, C.byref(hm.h), max_batch, max_seq, rank, world, buf, C.byref(h)))
        V = hm.h.vocab
        per = (V + world - 1) // world
        return cls(ctx, h, min(hm.h.n_layers, MAXL), V, max(1, min(per, V - rank * per)))

    def _ck(self, rc):
        return self.ctx.check(rc)

    def set_sampling(self, temperature, top_k):
        self._ck(lib().jdg_set_sampling(self.h, temperature, top_k))

    def reset(self, slot=-1):
        self._ck(lib().jdg_reset(self.h, slot))

    def set_prompt(self, tokens, lengths, rng=None):
        t = np.ascontiguousarray(tokens, np.int32)
        B, P = t.shape
        ln = np.ascontiguousarray(lengths, np.int32)
        r = None if rng is None else np.ascontiguousarray(rng, np.uint64)
        self._ck(lib().jdg_set_prompt(self.h, B, _p(t, I32P), P, _p(ln, I32P), None if r is None else _p(r, U64P)))

    def run(self, B, n_steps):
        self._ck(lib().jdg_run(self.h, B, n_steps))
        ms = C.c_float(0)
        lib().jdg_last_run_ms(self.h, C.byref(ms))
        return ms.value

    def host_learn(self, toks, lr, rng, offset):
        """Hebbian --learn pass over toks; returns (deaths, rng state, notorch offset)."""
        t = np.ascontiguousarray(toks, np.int32)
        st = np.array([rng], np.uint64)
        off = np.array([offset], np.int32)
        dead = np.zeros(1, np.int32)
        self._ck(lib().jdg_host_learn(self.h, _p(t, I32P), t.size, lr, _p(st, U64P), _p(off, I32P), _p(dead, I32P)))
        return int(dead[0]), int(st[0]), int(off[0])

    def expert(self, l, x, dim, rank):
        A = np.zeros((dim, rank), np.float32)
        B = np.zeros((rank, dim), np.float32)
        al = np.zeros(1, np.int32)
        self._ck(lib().jdg_host_get_expert(self.h, l, x, _p(A, F32P), _p(B, F32P), _p(al, I32P)))
        return A, B, int(al[0])

    def prefill(self, B):
        """Batched prompt prefill of slots 0..B-1 (after set_prompt); returns device ms."""
        self._ck(lib().jdg_prefill(self.h, B))
        ms = C.c_float(0)
        lib().jdg_last_run_ms(self.h, C.byref(ms))
        return ms.value

    def prefill_trace(self, n):
        """Elections of the last prefilled sequence's first n tokens, as trace arrays [n][L]."""
        t, d = self._trace_bufs(n)
        self._ck(lib().jdg_get_prefill_trace(self.h, n, C.byref(t)))
        return d

    def state(self, B):
        t = np.zeros(B, np.int32)
        p = np.zeros(B, np.int32)
        self._ck(lib().jdg_get_state(self.h, B, _p(t, I32P), _p(p, I32P)))
        return t, p

    def history(self, B, n):
        out = np.zeros((B, n), np.int32)
        self._ck(lib().jdg_get_history(self.h, B, n, _p(out, I32P)))
        return out

    def step(self, tok, pos, rng=None, logits=False, trace=False):
        tok = np.ascontiguousarray(tok, np.int32)
        pos = np.ascontiguousarray(pos, np.int32)
        B = tok.size
        nxt = np.zeros(B, np.int32)
        r = None if rng is None else np.ascontiguousarray(rng, np.uint64).copy()
        lg = np.zeros((B, self.ldl), np.float32) if logits else None
        tr, trd = (self._trace_bufs(B) if trace else (None, None))
        self._ck(lib().jdg_step(self.h, B, _p(tok, I32P), _p(pos, I32P), None if r is None else _p(r, U64P),
                                _p(nxt, I32P), None if lg is None else _p(lg, F32P),
                                C.byref(tr) if tr is not None else None))
        return nxt, r, lg, trd

    def _trace_bufs(self, B):
        d = {"k": np.zeros((B, self.L), np.int32), "sel": np.zeros((B, self.L, MAXE), np.int32),
             "w": np.zeros((B, self.L, MAXE), np.float32), "ema": np.zeros((B, self.L), np.float32)}
        t = JdgTrace(_p(d["k"], I32P), _p(d["sel"], I32P), _p(d["w"], F32P), _p(d["ema"], F32P))
        return t, d

    def logits(self, B):
        lg = np.zeros((B, self.ldl), np.float32)
        self._ck(lib().jdg_get_logits(self.h, B, _p(lg, F32P)))
        return lg

    def trace(self, B):
        t, d = self._trace_bufs(B)
        self._ck(lib().jdg_get_trace(self.h, B, C.byref(t)))
        return d

    def stats(self):
        """(experts read, KV positions read, steps) since reset_stats()."""
        out = np.zeros(3, np.uint64)
        self._ck(lib().jdg_get_stats(self.h, _p(out, U64P)))
        return int(out[0]), int(out[1]), int(out[2])

    def timeline(self, n_slots=0):
        """Arm (n_slots=0) or read the batch-1 kernel timeline as an [n_slots, 3] array (ns)."""
        out = np.zeros((max(n_slots, 1), 3), np.uint64)
        self._ck(lib().jdg_debug_timeline(self.h, n_slots, _p(out, U64P) if n_slots else None))
        return out[:n_slots]

    def reset_stats(self):
        self._ck(lib().jdg_reset_stats(self.h))

    def launches(self):
        n = C.c_longlong(0)
        lib().jdg_launch_count(self.h, C.byref(n))
        return n.value

    def close(self):
        if self.h:
            lib().jdg_engine_free(self.h)
            self.h = C.c_void_p()


def qmatvec(ctx, W, dt, x, r, c):
    """out[b][r] = W . x[b] on the GPU (x: [B][c] or [c])."""
    x = np.ascontiguousarray(x, np.float32)
    B = 1 if x.ndim == 1 else x.shape[0]
    out = np.zeros((B, r), np.float32)
    W = np.ascontiguousarray(W)
    ctx.check(lib().jdg_qmatvec(ctx.h, _p(out, F32P), W.ctypes.data_as(C.c_void_p), dt, _p(x, F32P), r, c, B))
    return out if x.ndim > 1 else out[0]
