"""Tensor-parallel host decode on 2 GPUs (one process per GPU, NCCL) against the oracle.

Heads, the FFN hidden slice and the vocabulary are split across the ranks; the all-reduced
residual must give the same logits (within the parity tolerance) and the same greedy stream
as the single-process oracle.  Skipped with fewer than 2 GPUs.
"""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

WORKER = r'''
import os, sys, json, ctypes as C
import numpy as np
sys.path.insert(0, os.path.join(sys.argv[5], "tests"))
import conftest
import janus_doe_b200 as jd
import torch, torch.distributed as dist
rank, world, path, out = int(sys.argv[1]), int(sys.argv[2]), sys.argv[3], sys.argv[4]
torch.cuda.set_device(rank)
dist.init_process_group("gloo", rank=rank, world_size=world)
hm = jd.HostModel(path, lora_rank=8)
hm.lora_seed(23, 4, 0.01, 1.0 / 512 ** 0.5)
ids = [None]
if rank == 0:
    buf = C.create_string_buffer(128)
    jd.check(jd.lib().jdg_comm_unique_id(buf))
    ids[0] = bytes(buf.raw)
dist.broadcast_object_list(ids, src=0)
ctx = jd.Context(rank)
eng = jd.Engine.host_tp(ctx, hm, 2, 64, rank, world, ids[0])
prompts = np.load(os.path.join(out, "prompts.npy"))
B, P = prompts.shape
eng.set_prompt(prompts, [P] * B)
eng.run(B, P - 1 + 12)
hist = eng.history(B, 12)
eng.reset()
lg_tp = []
stream = np.load(os.path.join(out, "stream.npy"))
for pos in range(stream.shape[1] - 1):
    _, _, lg, _ = eng.step(stream[:, pos], np.full(B, pos, np.int32), logits=True)
    lg_tp.append(lg.copy())
np.save(os.path.join(out, "hist%d.npy" % rank), hist)
np.save(os.path.join(out, "lg%d.npy" % rank), np.array(lg_tp))
eng.close(); ctx.close()
dist.barrier()
dist.destroy_process_group()
'''


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_tp2_matches_oracle(jd, orc, tmp_path):
    if jd.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from oracle.oracle import HostModel as OHost
    path = str(tmp_path / "tp.gguf")
    jd.write_synthetic_gguf(path, "llama", 2, 512, 1024, 8, 4, 1000, 5e5, 1e-5, 12, 17, 0.02)
    om = OHost(orc, path, 8, -1, 64)
    om.lora_seed(23, 4, 0.01, 1.0 / 512 ** 0.5)
    B, P, G = 2, 6, 12
    prompts = np.random.default_rng(4).integers(0, 1000, (B, P)).astype(np.int32)
    streams, logits = [], []
    for b in range(B):
        om.reset()
        st, lgs = list(prompts[b]), []
        for pos in range(P + G - 1):
            lo = om.forward(st[pos], pos)
            lgs.append(lo)
            if pos + 1 >= P:
                st.append(int(np.argmax(lo)))
        streams.append(st)
        logits.append(lgs)
    om.close()
    np.save(str(tmp_path / "prompts.npy"), prompts)
    np.save(str(tmp_path / "stream.npy"), np.array(streams, np.int32))
    wpath = str(tmp_path / "worker.py")
    open(wpath, "w").write(WORKER)
    env = dict(os.environ, MASTER_ADDR="127.0.0.1", MASTER_PORT=str(_free_port()), NCCL_NVLS_ENABLE="0")
    procs = [subprocess.Popen([sys.executable, wpath, str(r), "2", path, str(tmp_path), ROOT], env=env)
             for r in range(2)]
    for p in procs:
        assert p.wait(timeout=300) == 0
    hist = np.load(str(tmp_path / "hist0.npy"))
    assert np.array_equal(hist, np.load(str(tmp_path / "hist1.npy")))
    for b in range(B):
        assert list(hist[b]) == streams[b][P:], b
    # logits are vocabulary-sharded: rank r holds rows [r*500, r*500+500)
    lg = np.concatenate([np.load(str(tmp_path / "lg0.npy")), np.load(str(tmp_path / "lg1.npy"))], axis=-1)
    for b in range(B):
        for pos in range(P + G - 1):
            ref = logits[b][pos]
            err = np.max(np.abs(lg[pos, b, :1000] - ref)) / np.max(np.abs(ref))
            assert err <= 1e-3, (b, pos, err)
