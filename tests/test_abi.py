"""The C ABI and the host-side model code, on CPU (no GPU calls)."""
import ctypes as C
import os

import numpy as np
import pytest

from oracle.oracle import HostModel as OHost
from oracle.oracle import OwnModel


def test_library_exports_every_header_symbol(jd):
    lib = jd.lib()
    names = jd.exported_symbols()
    assert len(names) > 30
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


@pytest.mark.parametrize("depth", list(range(1, 33)))
def test_config_from_depth_matches_oracle(jd, orc, depth):
    a, b = jd.config_from_depth(depth), orc.config(depth)
    for f, _ in jd.JdConfig._fields_:
        assert getattr(a, f) == getattr(b, f), f


@pytest.mark.parametrize("depth,masks", [(2, False), (4, True), (6, True)])
def test_seeded_weights_match_oracle(jd, orc, depth, masks):
    cfg = jd.config_from_depth(depth, vocab_size=500, seq_len=32)
    pm = jd.Model.seeded(cfg, 9, 0.02, masks)
    om = OwnModel(orc, orc.config(depth, vocab_size=500, seq_len=32), 9, 0.02, masks)
    try:
        D, V, H = cfg.dim, cfg.vocab_size, cfg.hidden_dim
        assert np.array_equal(np.ctypeslib.as_array(pm.m.output, (V * D,)), np.ctypeslib.as_array(om.m.output, (V * D,)))
        for l in range(depth):
            assert pm.alive(l) == om.alive(l)
            for e in range(16):
                if pm.alive(l)[e]:
                    assert np.array_equal(np.ctypeslib.as_array(pm.m.layers[l].w_down[e], (D * H,)),
                                          np.ctypeslib.as_array(om.m.layers[l].w_down[e], (D * H,)))
    finally:
        om.close()


def test_own_gguf_roundtrip_and_rejects(jd, tmp_path):
    cfg = jd.config_from_depth(3, vocab_size=400, seq_len=32)
    m = jd.Model.seeded(cfg, 4, 0.02, True)
    path = str(tmp_path / "m.gguf")
    m.export_gguf(path)
    m2 = jd.Model(cfg)
    m2.load_gguf(path)
    D, V = cfg.dim, cfg.vocab_size
    assert np.array_equal(np.ctypeslib.as_array(m2.m.tok_emb, (V * D,)), np.ctypeslib.as_array(m.m.tok_emb, (V * D,)))
    assert [m2.alive(l) for l in range(3)] == [m.alive(l) for l in range(3)]
    # a different depth is not ours (janusdoe.c:1854-1857)
    other = jd.Model(jd.config_from_depth(4, vocab_size=400, seq_len=32))
    with pytest.raises(jd.JdError) as ei:
        other.load_gguf(path)
    assert ei.value.code == jd.JD_EFORMAT
    data = open(path, "rb").read()
    for cut in (3, 40, len(data) // 3, len(data) - 4):
        bad = str(tmp_path / ("cut%d.gguf" % cut))
        open(bad, "wb").write(data[:cut])
        with pytest.raises(jd.JdError):
            jd.Model(cfg).load_gguf(bad)
    bad = str(tmp_path / "magic.gguf")
    open(bad, "wb").write(b"XXXX" + data[4:])
    with pytest.raises(jd.JdError):
        jd.Model(cfg).load_gguf(bad)
    with pytest.raises(jd.JdError) as ei:
        jd.Model(cfg).load_gguf(str(tmp_path / "missing.gguf"))
    assert ei.value.code == jd.JD_EIO


@pytest.mark.parametrize("arch,dt,rope", [("llama", 8, 1), ("qwen2", 12, 0), ("mistral", 12, 1), ("gemma", 8, 0)])
def test_host_loader_matches_oracle(jd, orc, tmp_path, arch, dt, rope):
    path = str(tmp_path / "h.gguf")
    jd.write_synthetic_gguf(path, arch, 2, 512, 768, 8, 2, 900, 5e5, 1e-6, dt, 5, 0.02)
    hm = jd.HostModel(path, lora_rank=8)
    om = OHost(orc, path, 8, -1, 8)
    try:
        h, o = hm.h, om.h
        for f in ("n_layers", "dim", "hidden", "n_heads", "n_kv_heads", "head_dim", "vocab", "rope_norm"):
            assert getattr(h, f) == getattr(o, f), f
        assert h.rope_norm == rope and h.arch.decode() == arch
        assert abs(h.rope_theta - 5e5) < 1 and abs(h.rms_eps - 1e-6) < 1e-12
        assert np.array_equal(np.ctypeslib.as_array(h.tok_emb, (900 * 512,)), np.ctypeslib.as_array(o.tok_emb, (900 * 512,)))
        assert h.layers[1].wq_dt == dt and h.output_dt == dt
        # rope override flags (--rope-neox / --rope-norm)
        assert jd.HostModel(path, 8, rope_override=0).h.rope_norm == 0
        assert jd.HostModel(path, 8, rope_override=1).h.rope_norm == 1
    finally:
        om.close()
        hm.close()


def test_lora_seed_and_sidecar(jd, orc, tmp_path):
    path = str(tmp_path / "h.gguf")
    jd.write_synthetic_gguf(path, "llama", 2, 256, 256, 4, 4, 300, 1e4, 1e-6, 8, 5, 0.02)
    hm = jd.HostModel(path, lora_rank=16)
    hm.lora_seed(31, 6, 0.01, 0.1)
    om = OHost(orc, path, 16, -1, 8)
    om.lora_seed(31, 6, 0.01, 0.1)
    for l in range(2):
        assert np.array_equal(np.ctypeslib.as_array(hm.h.w_vote[l], (16 * 256,)), np.ctypeslib.as_array(om.h.w_vote[l], (16 * 256,)))
        for e in range(16):
            assert hm.h.alive[l][e] == (1 if e < 6 else 0)
        assert np.array_equal(np.ctypeslib.as_array(hm.h.B[l][5], (16 * 256,)), np.ctypeslib.as_array(om.h.B[l][5], (16 * 256,)))
    side = str(tmp_path / "lora.bin")
    hm.lora_save(side)
    hm2 = jd.HostModel(path, lora_rank=16)
    hm2.lora_load(side)
    for l in range(2):
        assert [hm2.h.alive[l][e] for e in range(16)] == [hm.h.alive[l][e] for e in range(16)]
        assert np.array_equal(np.ctypeslib.as_array(hm2.h.A[l][3], (256 * 16,)), np.ctypeslib.as_array(hm.h.A[l][3], (256 * 16,)))
    wrong = jd.HostModel(path, lora_rank=8)
    with pytest.raises(jd.JdError):
        wrong.lora_load(side)
    om.close()


def test_host_loader_rejects(jd, tmp_path):
    bad = str(tmp_path / "empty.gguf")
    open(bad, "wb").write(b"")
    with pytest.raises(jd.JdError):
        jd.HostModel(bad)
    with pytest.raises(jd.JdError):
        jd.HostModel(str(tmp_path / "nope.gguf"))
    with pytest.raises(jd.JdError):  # no essential tensors
        p = str(tmp_path / "hdr.gguf")
        import struct
        open(p, "wb").write(struct.pack("<IIQQ", 0x46554747, 3, 0, 0))
        jd.HostModel(p)


def test_synthetic_writer_rejects_bad_shapes(jd, tmp_path):
    with pytest.raises(jd.JdError):
        jd.write_synthetic_gguf(str(tmp_path / "x.gguf"), "llama", 1, 300, 256, 4, 4, 10, 1e4, 1e-6, 12, 1)
    with pytest.raises(jd.JdError) as ei:
        jd.write_synthetic_gguf(str(tmp_path / "x.gguf"), "llama", 1, 256, 256, 4, 4, 10, 1e4, 1e-6, 13, 1)
    assert ei.value.code == jd.JD_EUNSUPPORTED


@pytest.mark.parametrize("dt", [1, 2, 6, 14])
def test_synthetic_writer_other_types_match_oracle(jd, orc, tmp_path, dt):
    """Output heads in F16 / Q4_0 / Q5_0 / Q6_K: the product loader keeps them packed, and the
    oracle's decoder and the library's decoder give the same weights from the file."""
    import ctypes as C
    path = str(tmp_path / "m.gguf")
    jd.write_synthetic_gguf(path, "llama", 1, 512, 512, 8, 8, 300, 1e4, 1e-5, 8, 3, 0.02, out_dtype=dt)
    hm = jd.HostModel(path, lora_rank=8)
    om = OHost(orc, path, 8, -1, 8)
    try:
        assert hm.h.output_dt == dt and om.h.output_dt == dt
        rb = {1: 1024, 2: 16 * 18, 6: 16 * 22, 14: 2 * 210}[dt]
        W = np.frombuffer(C.string_at(hm.h.output, 300 * rb), np.uint8).copy()
        a, b = jd.dequant(W, 300 * 512, dt), orc.dequant(W, 300 * 512, dt)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
        assert 0.005 < float(np.std(a)) < 0.05   # the quantiser kept the N(0, 0.02) scale
    finally:
        om.close()
        hm.close()


def test_open_without_gpu_reports(jd):
    if jd.device_count() > 0:
        pytest.skip("a GPU is present")
    with pytest.raises(jd.JdError):
        jd.Context(0)


def _na_check(jd):
    f = jd.lib().jdg_logits_argmax_noalloc_check
    f.argtypes = [C.c_void_p] * 2 + [C.c_int] * 2 + [C.c_void_p] * 2
    f.restype = C.c_int
    return f


@pytest.mark.parametrize("W,x,rows,cols,code,msg", [
    (256, 512, 8256, 768, 0, None),                      # aligned, within the scratch
    (256, 512, 131072, 16384, 0, None),                  # the largest accepted call
    (256, 512, 131072 + 16, 64, -1, b"exceeds"),         # one CTA of rows past the scratch
    (256, 512, 64, 16384 + 4, -1, b"exceeds"),           # x no longer fits shared memory
    (256 + 4, 512, 64, 64, -1, b"16-byte aligned"),      # W view offset by one float
    (256, 512 + 8, 64, 64, -1, b"16-byte aligned"),      # x view offset by two floats
    (256, 512, 64, 66, -1, b"bad arguments"),            # cols not a multiple of 4
    (256, 512, 0, 64, -1, b"bad arguments"),             # no rows
    (0, 512, 64, 64, -1, b"bad arguments"),              # null W
])
def test_noalloc_argument_check(jd, W, x, rows, cols, code, msg):
    """Argument checks of the allocation-free pick, run on the host only: the values are
    plain integers standing in for device addresses and nothing is dereferenced."""
    rc = _na_check(jd)(W, x, rows, cols, 1024, 2048)
    assert rc == code
    if msg:
        assert msg in jd.lib().jdg_last_error(None)


@pytest.mark.parametrize("dt", [1, 2, 6, 8, 12, 14])
def test_product_dequant_matches_golden(jd, dt):
    """The loader's block decoder (jd_dequant) gives the reference's dequantised weights bit
    for bit for every GGUF type it reads (golden vectors from the reference build)."""
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "quant.npz"))
    if dt == 1:
        f16 = np.load(os.path.join(os.path.dirname(__file__), "golden", "f16.npz"))["bits"]
        halves = np.arange(65536, dtype=np.uint16)
        got = jd.dequant(halves.view(np.uint8), 65536, 1).view(np.uint32)
        # the fixture's values went through a C float return and a Python float, which sets the
        # quiet bit of a signalling NaN; compare NaN payloads with that bit masked
        nan = (f16 & 0x7F800000) == 0x7F800000
        nan &= (f16 & 0x007FFFFF) != 0
        assert np.array_equal(got[~nan], f16[~nan])
        assert np.array_equal(got[nan] | 0x00400000, f16[nan] | 0x00400000)
        return
    W, ref = g["W%d" % dt], g["dq%d" % dt]
    got = jd.dequant(W.reshape(-1), ref.size, dt)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_product_dequant_rejects_unknown_type(jd):
    with pytest.raises(jd.JdError) as ei:
        jd.dequant(np.zeros(64, np.uint8), 32, 3)
    assert ei.value.code == jd.JD_EUNSUPPORTED


def test_host_tokenizer_matches_reference(jd, tmp_path):
    """Whole-word tokenisation and token printing (janusdoe.c:3329-3356) against the reference
    build on the synthetic vocabulary: "Ġword" and "word" forms, repeated texts (lowest id),
    unknown words spelled byte by byte, bytes without a token, words beyond 120 bytes, runs of
    spaces, and the id limit."""
    from oracle.oracle import Reference
    try:
        ref = Reference("")
    except RuntimeError:
        pytest.skip("reference build absent")
    path = str(tmp_path / "tok.gguf")
    jd.write_synthetic_gguf(path, "llama", 1, 256, 512, 4, 2, 3000, 1e4, 1e-5, 8, 3, 0.02)
    hm = jd.HostModel(path, lora_rank=8)
    ref.host_load(path)
    try:
        V = 3000
        words = [hm.token_text(i).strip() for i in range(98, V, 7)]
        texts = [b"", b"   ", b"a", b" ".join(words[:40]), b"  " + b"   ".join(words[40:80]) + b"  ",
                 b"zzqqy xylophone " + words[3], "café naïve 日本".encode(),
                 b"k" * 150 + b" " + words[5], b"!@# $%^ &*()", b"<s> </s> <unk>",
                 b" ".join(words[80:]), b"x" * 121, bytes(range(32, 127))]
        texts += [hm.token_text(i).strip() for i in range(400, V, 997)]
        for t in texts:
            for mx in (256, 5):
                assert hm.tokenize(t, mx) == ref.host_tokenize(t, mx), (t[:60], mx)
        assert hm.tokenize(b"anything", 0) == []
        for i in list(range(-2, 120)) + list(range(120, V, 13)) + [V - 1, V, V + 5]:
            assert hm.token_text(i) == ref.host_decode_print(i), i
        # repeated texts resolve to the lowest id
        for i in range(500, V, 997):
            assert hm.tokenize(hm.token_text(i).strip() or b"?") == ref.host_tokenize(hm.token_text(i).strip() or b"?")
    finally:
        hm.close()
        ref.lib.jdr_host_free()
