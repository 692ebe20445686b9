"""Shared helpers for the parity tests: synthetic workloads and the comparison rules.

Rules (from the parity contract):
  * logits: max|gpu - ref| <= LOGIT_TOL * max|ref| per step (norm-relative);
  * elections (k and the elected slots in order) and greedy tokens: identical, except
    where the reference itself sits on a near-tie (reported, then re-synchronised).
"""
import numpy as np

LOGIT_TOL = 1e-3     # norm-relative logit tolerance
EMA_TOL = 1e-5       # absolute tolerance on the consensus EMA
TIE_LOGIT = 1e-4     # relative top-2 logit gap below which a greedy pick is a near-tie
TIE_VOTE = 1e-5      # relative vote gap below which an election is a near-tie
TIE_K = 1e-4         # n*(1-EMA) within this of an integer is a near-tie for k


def logit_err(gpu, ref):
    return float(np.max(np.abs(gpu - ref)) / max(1e-30, float(np.max(np.abs(ref)))))


def greedy_near_tie(ref_logits):
    s = np.sort(ref_logits)
    return (s[-1] - s[-2]) <= TIE_LOGIT * max(1e-30, abs(s[-1]))


def election_near_tie(tr_ref, l, n_alive):
    """Near-tie in layer l of a reference trace dict (from the oracle)."""
    ema = float(tr_ref["ema"][l])
    kf = n_alive * (1.0 - ema)
    if abs(kf - round(kf)) < TIE_K:
        return True
    return False


def compare_trace(gpu_tr, ref_tr, L, b=0):
    """Return list of (layer, what) mismatches between a GPU trace (batch index b) and an
    oracle trace for one step."""
    bad = []
    for l in range(L):
        k = int(ref_tr["k"][l])
        if int(gpu_tr["k"][b, l]) != k:
            bad.append((l, "k %d vs %d" % (gpu_tr["k"][b, l], k)))
            continue
        if list(gpu_tr["sel"][b, l, :k]) != list(ref_tr["sel"][l, :k]):
            bad.append((l, "sel %s vs %s" % (list(gpu_tr["sel"][b, l, :k]), list(ref_tr["sel"][l, :k]))))
        if abs(float(gpu_tr["ema"][b, l]) - float(ref_tr["ema"][l])) > EMA_TOL:
            bad.append((l, "ema %.8f vs %.8f" % (gpu_tr["ema"][b, l], ref_tr["ema"][l])))
        if k and np.max(np.abs(gpu_tr["w"][b, l, :k] - ref_tr["w"][l, :k])) > 1e-4:
            bad.append((l, "w"))
    return bad
