"""The `m` command line on the GPU against the oracle: own-model chat at depth 4 (byte
tokens, greedy) and --host generation on a synthetic GGUF (BOS + whole-word tokenisation,
greedy with the LoRA parliament, stop at EOS).  The binary prints its token ids with
--print-ids; they must equal the oracle's stream from the same prompt."""
import os
import subprocess

import numpy as np
import pytest

from oracle.oracle import HostModel as OHost
from oracle.oracle import OwnModel

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
M = os.path.join(ROOT, "janus.doe_b200", "m")


def _run_m(args):
    r = subprocess.run([M] + args, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr + r.stdout
    ids = {}
    for line in r.stdout.splitlines():
        if line.startswith("[ids] "):
            parts = line.split()
            ids[parts[1]] = [int(t) for t in parts[2:]]
    return ids, r.stdout


def test_m_depth4_greedy(orc):
    """m --depth 4 (seeded weights, seed 0) greedy from a byte prompt."""
    ask, gen = "The capital of France is", 24
    ids, out = _run_m(["--depth", "4", "--ask", ask, "--gen", str(gen), "--temp", "0", "--print-ids"])
    prompt = [b for b in ask.encode()]
    assert ids["prompt"] == prompt
    cfg = orc.config(4)
    om = OwnModel(orc, cfg, 0, 0.02, False)
    try:
        lg = None
        for pos, t in enumerate(prompt):
            lg = om.forward(t, pos)
        exp, pos = [], len(prompt)
        for _ in range(gen):
            nxt = int(np.argmax(lg))
            if nxt == 257:
                break
            exp.append(nxt)
            lg = om.forward(nxt, pos)
            pos += 1
    finally:
        om.close()
    assert ids["generated"] == exp, out


def test_m_host_greedy(jd, orc, tmp_path):
    """m --host on a synthetic Q4_K llama GGUF: the prompt ids are BOS + the reference's
    tokenisation, the generated ids the oracle's greedy stream (LoRA parliament drawn from
    --seed as the CLI does: 4 adapters, A/B std 0.005, vote amplitude 0.02)."""
    path = str(tmp_path / "cli.gguf")
    jd.write_synthetic_gguf(path, "llama", 2, 512, 1024, 8, 2, 3000, 5e5, 1e-5, 12, 41, 0.02)
    hm = jd.HostModel(path, lora_rank=8)
    words = [hm.token_text(i).strip().decode() for i in (140, 377, 901, 1513)]
    hm.close()
    ask = " ".join(words) + " zq"
    gen, seed = 12, 5
    ids, out = _run_m(["--host", path, "--ask", ask, "--gen", str(gen), "--seed", str(seed), "--lora-rank", "8",
                       "--print-ids"])
    hm = jd.HostModel(path, lora_rank=8)
    try:
        exp_prompt = [1] + hm.tokenize(ask, 200)
    finally:
        hm.close()
    assert ids["prompt"] == exp_prompt
    om = OHost(orc, path, 8, -1, 256)
    om.lora_seed(seed, 4, 0.02 / 4.0, 0.02)
    try:
        lg = None
        for pos, t in enumerate(exp_prompt):
            lg = om.forward(t, pos)
        exp, pos = [], len(exp_prompt)
        for _ in range(gen):
            nxt = int(np.argmax(lg))
            if nxt == 2:
                break
            exp.append(nxt)
            lg = om.forward(nxt, pos)
            pos += 1
    finally:
        om.close()
    assert ids["generated"] == exp, out
