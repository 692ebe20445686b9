"""Decode throughput of the janus.DoE token loop on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

One "step" is one decode step of the whole batch (one token per sequence) after a
sequential prefill of the prompt.  Without --workload the run measures depth12_bs256, then
host_q4k_bs32, then depth12_bs1, and prints one JSON line per workload, the depth12_bs1
headline last (K and W apply to the headline; the others take at most their own defaults).
Workloads (synthetic seeded weights, uniform-random prompts):
  depth12_bs1    (default) own model depth 12 (dim 768, 12/4 heads, 8 experts with 5-8 alive
                 per layer, vocab 8256, ctx 1024), 512-token prompt, greedy, batch 1 per GPU
  depth12_bs256  same model, 256 sequences per GPU
  depth4_bs1     depth 4 (dim 256, 4 experts, vocab 2256), 32-token prompt, greedy
  depth8_bs64    depth 8 (dim 512, 8/4 heads, 6 experts, vocab 4256), 64 sequences,
                 64-token prompt, temperature 0.8 / top-k 40
  host_q8_bs1    host GGUF, Q8_0, 1.1B llama shape (dim 2048, 22 layers), batch 1
  host_q4k_bs32  host GGUF, Q4_K, 8B llama shape (dim 4096, 32 layers, vocab 128256), 32 sequences
Own-model sequences are independent, so N GPUs each run their own batch (weak scaling, no
collective); the host model's 32 sequences are split over N GPUs by tensor parallelism with
NCCL all-reduces (strong scaling).
`value` is device-timed (CUDA events on the engine's stream, max over ranks); `e2e` goes
through the public step call with host buffers (pinned H2D of token/position, D2H of the
next token every step).
"""
import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
METRIC = "decode tok/s (bs1, bs256) depth-12 & host Q4_K 8B; % of HBM roofline"

WORKLOADS = {
    "depth12_bs1": dict(depth=12, over=dict(n_kv_heads=4, vocab_size=8256, seq_len=1024), masks=True, seed=2,
                        B=1, prompt=512, temp=0.0, top_k=0, steps=256, warmup=8, ref_decode=64),
    "depth12_bs256": dict(depth=12, over=dict(n_kv_heads=4, vocab_size=8256, seq_len=1024), masks=True, seed=2,
                          B=256, prompt=512, temp=0.0, top_k=0, steps=32, warmup=4, ref_decode=8),
    "depth4_bs1": dict(depth=4, over=dict(vocab_size=2256, seq_len=256), masks=False, seed=0,
                       B=1, prompt=32, temp=0.0, top_k=0, steps=128, warmup=8, ref_decode=128,
                       l2="model L2-resident (16 MB of weights): tok/s and latency, no HBM claim"),
    "depth8_bs64": dict(depth=8, over=dict(n_kv_heads=4, vocab_size=4256, seq_len=512), masks=False, seed=1,
                        B=64, prompt=64, temp=0.8, top_k=40, steps=128, warmup=8, ref_decode=32),
    # host GGUF mode: synthetic llama-family models, weights N(0, 0.02) quantised per block
    "host_q8_bs1": dict(host=True, arch="qwen2", L=22, D=2048, H=32, KV=4, FF=5632, V=32000, dtype=8, theta=1e4,
                        rank=8, adapters=4, seed=3, B=1, prompt=64, max_seq=320, steps=128, warmup=8,
                        ref_prompt=8, ref_decode=8, temp=0.0, top_k=0),
    "host_q4k_bs32": dict(host=True, arch="llama", L=32, D=4096, H=32, KV=8, FF=14336, V=128256, dtype=12,
                          theta=5e5, rank=16, adapters=8, seed=4, B=32, prompt=128, max_seq=384, steps=32, warmup=4,
                          ref_prompt=4, ref_decode=4, temp=0.0, top_k=0),
}


def load_pkg():
    import importlib.util
    name = "janus_doe_b200"
    if name in sys.modules:
        return sys.modules[name]
    pkg = os.path.join(ROOT, "janus.doe_b200")
    spec = importlib.util.spec_from_file_location(name, os.path.join(pkg, "__init__.py"),
                                                  submodule_search_locations=[pkg])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def dram_traffic(workload, alg_bytes_per_step):
    """DRAM bytes per step from an ncu capture of this workload (profiles/dram_traffic.json):
    the captured traffic/algorithmic ratio applied to this run's algorithmic bytes."""
    p = os.path.join(ROOT, "profiles", "dram_traffic.json")
    if os.path.exists(p):
        d = json.load(open(p))
        if workload in d:
            return d[workload]["traffic_over_algorithmic"] * alg_bytes_per_step
    return None


class Clocks:
    """SM clock and throttle reasons sampled during the timed region: NVML polled every 2 ms
    from a thread (so even a region of a few milliseconds gets samples), nvidia-smi at 200 ms
    when NVML is not importable."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, gpu_index):
        self.idx, self.rows, self.proc, self.nv = gpu_index, [], None, None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(gpu_index)
            self.bits = [pynvml.nvmlClocksEventReasonHwSlowdown, pynvml.nvmlClocksEventReasonHwThermalSlowdown,
                         pynvml.nvmlClocksEventReasonSwThermalSlowdown, pynvml.nvmlClocksEventReasonSwPowerCap]
        except Exception:
            self.nv = None

    def _poll(self):
        nv = self.nv
        while not self.done:
            try:
                self.samples.append((nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM),
                                     nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)))
            except Exception:
                pass
            time.sleep(0.002)

    def start(self):
        if self.nv is not None:
            self.samples, self.done = [], False
            self.th = threading.Thread(target=self._poll, daemon=True)
            self.th.start()
            t0 = time.time()
            while not self.samples and time.time() - t0 < 2.0:  # the first sample precedes the region
                time.sleep(0.001)
            self.n0 = len(self.samples)
            return
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.idx), "--query-gpu=" + self.Q,
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.th = threading.Thread(target=self._read, daemon=True)
            self.th.start()
        except (OSError, FileNotFoundError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def stop(self):
        if self.nv is not None:
            self.done = True
            self.th.join(timeout=1.0)
            inside = self.samples[self.n0:] or self.samples[-1:]
            sm = [float(c) for c, _ in inside]
            reasons = sorted({self.NAMES[i] for _, r in inside for i, b in enumerate(self.bits) if r & b})
            try:
                mx = float(self.nv.nvmlDeviceGetMaxClockInfo(self.h, self.nv.NVML_CLOCK_SM))
            except Exception:
                mx = None
            return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": reasons,
                    "samples": len(sm), "source": "nvml, 2 ms"}
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm = [float(r[1]) for r in self.rows if len(r) >= 8 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if len(r) >= 8 and r[2].replace(".", "").isdigit()]
        reasons = sorted({self.NAMES[i] for r in self.rows if len(r) >= 8 for i in range(4) if r[4 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(sm), "source": "nvidia-smi, 200 ms"}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world == 1:
        return None, 1, 0, 0
    import datetime

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    return dist, world, rank, local


def barrier(dist):
    if dist is not None:
        import torch
        dist.barrier()
        torch.cuda.synchronize()


def allmax(dist, v):
    """Max of a host float over ranks (device tensor under NCCL, host tensor under gloo)."""
    if dist is None:
        return v
    import torch
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def prompts_for(w, rank):
    """Uniform-random prompt ids per sequence from splitmix64(seed*1000 + s)."""
    V = w["over"]["vocab_size"]
    B, P = w["B"], w["prompt"]
    out = np.zeros((B, P), np.int32)
    rngs = np.zeros(B, np.uint64)
    for b in range(B):
        s = w["seed"] * 1000 + rank * B + b
        x = _splitmix(s)
        for i in range(P):
            x = _xs(x)
            out[b, i] = x % V
        rngs[b] = x
    return out, rngs


M64 = (1 << 64) - 1


def _splitmix(x):
    z = (x + 0x9E3779B97F4A7C15) & M64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M64
    z = z ^ (z >> 31)
    return z or 1


def _xs(x):
    x ^= (x << 13) & M64
    x ^= x >> 7
    x ^= (x << 17) & M64
    return x & M64


def own_bytes(cfg, alive_counts, B, steps, stats):
    """Algorithmic HBM bytes of `steps` decode steps (f32 weights and KV):
    per step every attention matrix, norm and alive vote row, the LM head, the gathered
    embedding rows; per (step, layer) the experts read (union over the batch, counted on
    the device); KV read (sum of pos+1 over sequences, counted on the device) + append."""
    D, H, V, L = cfg.dim, cfg.hidden_dim, cfg.vocab_size, cfg.depth
    qd, kd = cfg.n_heads * cfg.head_dim, cfg.n_kv_heads * cfg.head_dim
    fixed = 4 * (V * D + D + B * D)
    for l in range(L):
        fixed += 4 * (2 * D + (qd + 2 * kd) * D + D * qd + alive_counts[l] * D)
    experts, kvpos, nsteps = stats
    return steps * fixed + experts * 3 * H * D * 4 + kvpos * L * 2 * kd * 4 + steps * B * L * 2 * kd * 4


def cpu_reference(w, n_decode, threads):
    """Time the reference's own decode (janusdoe.c forward_token + greedy/sample, OpenBLAS
    build from oracle/_ref) on the host cores: one sequence, prefill untimed, n_decode
    decode tokens timed.  Returns (tok/s, kind, sample text, alive experts per layer)."""
    os.environ["OPENBLAS_NUM_THREADS"] = str(threads)
    sys.path.insert(0, ROOT)
    from oracle.oracle import Reference
    try:
        ref = Reference("_blas")
    except RuntimeError:
        ref = Reference("")
    kind = "reference"
    ov = w["over"]
    ref.own_setup(w["depth"], ov.get("n_kv_heads", 0), ov["vocab_size"], ov.get("seq_len", 256), w["seed"], 0.02,
                  w["masks"])
    alive = [int(sum(ref.own_alive(l))) for l in range(w["depth"])]
    pr, rngs = prompts_for(dict(w, B=1), 0)
    pos, lg = 0, None
    for t in pr[0]:
        lg, _ = ref.own_forward(int(t), pos)
        pos += 1
    st = int(rngs[0])
    t0 = time.perf_counter()
    for _ in range(n_decode):
        if w["temp"] > 0:
            nxt, st = ref.sample(lg, w["temp"], w["top_k"], st)
        else:
            nxt = int(np.argmax(lg))
        lg, _ = ref.own_forward(nxt, pos)
        pos += 1
    dt = time.perf_counter() - t0
    return n_decode / dt, kind, "1 sequence, %d-token prefill untimed, %d decode tokens timed (positions %d-%d)" % (
        w["prompt"], n_decode, w["prompt"], w["prompt"] + n_decode - 1), alive


def host_gguf_path(w):
    """Synthetic GGUF of a host workload, generated once per machine (all cores)."""
    d = os.environ.get("JD_BENCH_DIR", "/tmp")
    return os.path.join(d, "jd_%s_L%d_D%d_V%d_s%d.gguf" % (w["arch"], w["L"], w["D"], w["V"], w["seed"]))


def ensure_host_gguf(jd, w):
    path = host_gguf_path(w)
    if not os.path.exists(path):
        tmp = path + ".part%d" % os.getpid()
        jd.write_synthetic_gguf(tmp, w["arch"], w["L"], w["D"], w["FF"], w["H"], w["KV"], w["V"], w["theta"], 1e-5,
                                w["dtype"], w["seed"], 0.02, 0)
        os.replace(tmp, path)
    return path


def lora_args(w):
    # A, B ~ N(0, 0.01); vote rows uniform in [-1/sqrt(D), 1/sqrt(D))
    return w["seed"] * 7 + 1, w["adapters"], 0.01, 1.0 / w["D"] ** 0.5


def cpu_reference_host(w, n_prompt, n_decode):
    """The reference's gguf_host_forward (its own pthread row kernels, janusdoe.c:2685) on the
    host cores: one sequence, n_prompt prompt tokens untimed, n_decode greedy tokens timed."""
    sys.path.insert(0, ROOT)
    from oracle.oracle import Reference
    jd = load_pkg()
    path = ensure_host_gguf(jd, w)
    ref = Reference("_r8" if w["rank"] == 8 else "")
    ref.host_load(path)
    ref.lib.jdr_host_lora_seed(*lora_args(w))
    ref.lib.jdr_host_reset_seq(n_prompt + n_decode + 1)
    pr, _ = prompts_for(dict(w, B=1, over=dict(vocab_size=w["V"]), prompt=n_prompt), 0)
    lg = None
    for pos, t in enumerate(pr[0]):
        lg, _ = ref.host_forward(int(t), pos)
    pos = n_prompt
    t0 = time.perf_counter()
    for _ in range(n_decode):
        lg, _ = ref.host_forward(int(np.argmax(lg)), pos)
        pos += 1
    dt = time.perf_counter() - t0
    ref.lib.jdr_host_free()
    threads = min(32, os.cpu_count() or 1)
    return n_decode / dt, threads, "1 sequence, %d-token prompt untimed, %d greedy tokens timed" % (n_prompt, n_decode)


def own_config(name, w, world, alive, steps, warmup):
    """The workload description printed by both arms (identical for the same command line)."""
    ov = w["over"]
    P = w["prompt"]
    # config_from_depth: dim = 64 * depth, heads of 64
    return {"workload": name, "depth": w["depth"], "dim": 64 * w["depth"], "heads": w["depth"],
            "kv_heads": ov.get("n_kv_heads") or w["depth"], "experts_alive": alive, "vocab": ov["vocab_size"],
            "ctx": ov.get("seq_len"), "batch_per_gpu": w["B"], "global_batch": w["B"] * world, "prompt": P,
            "positions": [P + warmup, P + warmup + steps - 1],
            "sampling": "greedy" if w["temp"] <= 0 else "temp %.1f top-k %d" % (w["temp"], w["top_k"]),
            "parallelism": "dp%d (independent sequences)" % world,
            "l2": w.get("l2", "inputs larger than L2 (weights + KV read per step > 126 MB)")}


def host_config(name, w, world):
    return {"workload": name, "arch": w["arch"], "layers": w["L"], "dim": w["D"], "heads": w["H"],
            "kv_heads": w["KV"], "ffn": w["FF"], "vocab": w["V"], "dtype": {8: "Q8_0", 12: "Q4_K"}[w["dtype"]],
            "lora": "%d x rank %d" % (w["adapters"], w["rank"]), "global_batch": w["B"], "prompt": w["prompt"],
            "parallelism": "tp%d" % world if world > 1 else "1 GPU",
            "l2": "inputs larger than L2 (packed weights read per step > 126 MB)"}


def scaling_of(w):
    # own model: every GPU decodes its own batch (weak); host model: one batch of 32 sequences
    # split by tensor parallelism over the GPUs (strong)
    return "strong" if w.get("host") else "weak"


def reference_line(args, name, w, steps, warmup):
    """The reference arm for one workload: the reference's own CPU decode (rank 0 only)."""
    threads = os.cpu_count() or 1
    if w.get("host"):
        tps, threads, sample = cpu_reference_host(w, w["ref_prompt"], w["ref_decode"])
        cfg = host_config(name, w, args.gpus)
    else:
        n = max(1, min(steps, w["ref_decode"] * 4))
        tps, _, sample, alive = cpu_reference(w, n, threads)
        cfg = own_config(name, w, args.gpus, alive, steps, warmup)
    return {"impl": "reference", "metric": METRIC, "value": tps, "unit": "tok/s", "n_gpus": args.gpus,
            "steps": steps, "warmup": warmup, "ms_per_step": 1000.0 / tps, "higher_is_better": True,
            "scaling": scaling_of(w), "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": cfg,
            "cpu_baseline": {"value": tps, "unit": "tok/s", "cores": threads, "kind": "reference", "sample": sample},
            "e2e": {"value": tps, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def packed_bytes(w):
    """Packed weight bytes of a host model (per weight: 34/32 B for Q8_0, 144/256 B for Q4_K)."""
    bpw = {8: 34 / 32, 12: 144 / 256, 0: 4}[w["dtype"]]
    D, FF, V, L = w["D"], w["FF"], w["V"], w["L"]
    hd = D // w["H"]
    per_layer = (w["H"] * hd + 2 * w["KV"] * hd) * D + D * w["H"] * hd + 3 * FF * D
    return bpw * (L * per_layer + V * D)


def run_host(args, name, w, steps, warmup, dist, world, rank, local):
    jd = load_pkg()
    B, P, S = w["B"], w["prompt"], w["max_seq"]
    if rank == 0:
        ensure_host_gguf(jd, w)
    barrier(dist)
    path = ensure_host_gguf(jd, w)
    hm = jd.HostModel(path, lora_rank=w["rank"])
    hm.lora_seed(*lora_args(w))
    ctx = jd.Context(local)
    if world > 1:
        ids = [None]
        if rank == 0:
            buf = C.create_string_buffer(128)
            jd.check(jd.lib().jdg_comm_unique_id(buf))
            ids[0] = bytes(buf.raw)
        dist.broadcast_object_list(ids, src=0)
        eng = jd.Engine.host_tp(ctx, hm, B, S, rank, world, ids[0])
    else:
        eng = jd.Engine.host(ctx, hm, B, S)
    prompts, _ = prompts_for(dict(w, over=dict(vocab_size=w["V"])), 0)
    eng.set_prompt(prompts, [P] * B)
    prefill_ms = eng.run(B, P - 1)
    eng.run(B, warmup)
    clocks = Clocks(local)
    barrier(dist)
    eng.reset_stats()
    l0 = eng.launches()
    clocks.start()
    ms = eng.run(B, steps)
    ck = clocks.stop()
    n_launch = eng.launches() - l0
    stats = eng.stats()
    ms = allmax(dist, ms)
    barrier(dist)
    value = B * steps / (ms / 1000.0)
    n_e2e = min(steps, 16)
    tok_h, pos_h = eng.state(B)
    barrier(dist)
    t0 = time.perf_counter()
    for _ in range(n_e2e):
        nxt, _, _, _ = eng.step(tok_h, pos_h)
        tok_h, pos_h = nxt, pos_h + 1
    e2e_s = allmax(dist, time.perf_counter() - t0)
    barrier(dist)
    tr = eng.trace(B)
    # algorithmic bytes per step: packed weights (each rank reads its shard), f32 tok_emb rows,
    # the LoRA factors and vote rows of the experts elected by any sequence (last step's trace)
    # in every layer, KV read (device count) + append
    L, D, R = w["L"], w["D"], w["rank"]
    kd = w["KV"] * (D // w["H"])
    lora = 0
    for l in range(L):
        used = {int(e) for b in range(B) for e in tr["sel"][b, l] if e >= 0}
        lora += len(used) * 2 * D * R * 4 + w["adapters"] * D * 4
    per_step = packed_bytes(w) + B * D * 4 + world * lora + 4 * D * (2 * L + 1)
    bytes_run = steps * per_step + stats[1] * L * 2 * kd * 4 + steps * B * L * 2 * kd * 4
    peak, peak_kind = peaks()
    achieved = bytes_run / (ms / 1000.0) / 1e9
    roof = {"bound": "hbm", "achieved": achieved, "peak": peak * world, "unit": "GB/s",
            "frac": achieved / (peak * world), "traffic": dram_traffic(name, bytes_run / steps),
            "peak_source": peak_kind,
            "kernel": "whole decode step (CUDA graph of %d launches)" % (n_launch // max(1, steps)),
            "algorithmic_bytes_per_step": bytes_run / steps}
    line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": steps,
            "warmup": warmup, "ms_per_step": ms / steps, "higher_is_better": True,
            "scaling": scaling_of(w), "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (GGUF of N(0,0.02) weights quantised per block, uniform prompts)",
            "config": host_config(name, w, world),
            "roofline": roof, "prefill_ms": prefill_ms, "clocks": ck, "gpu_launches": n_launch,
            "e2e": {"value": B * n_e2e / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": 8 * B,
                    "d2h_bytes_per_step": 4 * B, "steps": n_e2e}}
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        tps, threads, sample = cpu_reference_host(w, w["ref_prompt"], w["ref_decode"])
        line["cpu_baseline"] = {"value": tps, "unit": "tok/s", "cores": threads, "kind": "reference",
                                "sample": sample}
    eng.close()
    hm.close()
    ctx.close()
    return line if rank == 0 else None


def run_own(args, name, w, steps, warmup, dist, world, rank, local):
    jd = load_pkg()
    B, P = w["B"], w["prompt"]
    cfg = jd.config_from_depth(w["depth"], **w["over"])
    ctx = jd.Context(local)
    model = jd.Model.seeded(cfg, w["seed"], 0.02, w["masks"])
    alive = [sum(model.alive(l)) for l in range(cfg.depth)]
    eng = jd.Engine.own(ctx, model, B)
    eng.set_sampling(w["temp"], w["top_k"])
    prompts, rngs = prompts_for(w, rank)
    # prompt prefill, timed separately: one sequence runs its prompt as one batch of tokens
    # (jdg_prefill); a batch of sequences runs it position by position as batched steps
    eng.set_prompt(prompts, [P] * B, rngs)
    prefill_ms = eng.prefill(B) if B == 1 else eng.run(B, P - 1)
    # warm-up decode steps
    eng.run(B, warmup)
    # timed decode steps
    clocks = Clocks(local)
    barrier(dist)
    eng.reset_stats()
    l0 = eng.launches()
    clocks.start()
    ms = eng.run(B, steps)
    ck = clocks.stop()
    n_launch = eng.launches() - l0
    stats = eng.stats()
    ms = allmax(dist, ms)
    barrier(dist)
    tok = B * steps * world
    value = tok / (ms / 1000.0)
    # e2e through the public step call with host buffers
    n_e2e = min(steps, 64)
    tok_h, pos_h = eng.state(B)
    rng_h = None if w["temp"] <= 0 else np.array(rngs, np.uint64)
    barrier(dist)
    t0 = time.perf_counter()
    for _ in range(n_e2e):
        nxt, rng_h, _, _ = eng.step(tok_h, pos_h, rng=rng_h)
        tok_h = nxt
        pos_h = pos_h + 1
    e2e_s = allmax(dist, time.perf_counter() - t0)
    barrier(dist)
    e2e = B * n_e2e * world / e2e_s
    # roofline: algorithmic bytes per step / device time per step (the decode step graph)
    bytes_run = own_bytes(cfg, alive, B, steps, stats)
    peak, peak_kind = peaks()
    achieved = bytes_run / (ms / 1000.0) / 1e9
    traffic = dram_traffic(name, bytes_run / steps)
    roof = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
            "traffic": traffic, "peak_source": peak_kind,
            "kernel": "whole decode step (CUDA graph of %d launches)" % (n_launch // max(1, steps)),
            "algorithmic_bytes_per_step": bytes_run / steps}
    line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": steps,
            "warmup": warmup, "ms_per_step": ms / steps, "higher_is_better": True, "scaling": scaling_of(w),
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,0.02) weights, uniform prompts)",
            "config": own_config(name, w, world, alive, steps, warmup),
            "roofline": roof, "prefill_ms": prefill_ms, "clocks": ck, "gpu_launches": n_launch,
            "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 8 * B, "d2h_bytes_per_step": 4 * B,
                    "steps": n_e2e}}
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        tps, kind, sample, _ = cpu_reference(w, w["ref_decode"], threads)
        line["cpu_baseline"] = {"value": tps, "unit": "tok/s", "cores": threads, "kind": kind, "sample": sample}
    eng.close()
    model.close()
    ctx.close()
    return line if rank == 0 else None


# The default run (no --workload) measures the three workloads the metric names and prints
# one JSON line each; the batch-1 depth-12 line, the headline, comes last.
DEFAULT_RUN = ["depth12_bs256", "host_q4k_bs32", "depth12_bs1"]


def steps_for(args, name, w, headline):
    """Timed steps and warm-up steps of one workload: the command line's K and W for the
    headline workload, at most the workload's own defaults for the others; bounded so that
    prompt + warm-up + timed + end-to-end steps fit the context."""
    if headline:
        steps = w["steps"] if args.steps is None else args.steps
        warmup = w["warmup"] if args.warmup is None else max(3, args.warmup)
    else:
        steps = w["steps"] if args.steps is None else min(args.steps, w["steps"])
        warmup = w["warmup"] if args.warmup is None else max(3, min(args.warmup, w["warmup"]))
    ctx = w["max_seq"] if w.get("host") else w["over"]["seq_len"]
    e2e = 16 if w.get("host") else 64
    if w["prompt"] + warmup + steps + min(steps, e2e) + 1 > ctx:
        steps = max(1, (ctx - w["prompt"] - warmup - 2) * 2 // 3)
    return steps, warmup


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=None)
    ap.add_argument("--workload", default=None, choices=sorted(WORKLOADS),
                    help="one workload only (default: %s, the last being the headline)" % ", ".join(DEFAULT_RUN))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--prompt", type=int, default=None, help="override the prompt length (profiling runs)")
    args = ap.parse_args()
    names = [args.workload] if args.workload else DEFAULT_RUN
    dist, world, rank, local = (None, 1, int(os.environ.get("RANK", "0")), 0) if args.impl == "reference" \
        else dist_setup()
    for i, name in enumerate(names):
        w = dict(WORKLOADS[name])
        if args.prompt:
            w["prompt"] = max(2, args.prompt)
        steps, warmup = steps_for(args, name, w, i == len(names) - 1)
        if args.impl == "reference":
            # the reference is one CPU process: rank 0 runs it, other ranks exit without work
            line = reference_line(args, name, w, steps, warmup) if rank == 0 else None
        elif w.get("host"):
            line = run_host(args, name, w, steps, warmup, dist, world, rank, local)
        else:
            line = run_own(args, name, w, steps, warmup, dist, world, rank, local)
        if line is not None:
            print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
