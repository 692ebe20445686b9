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


def _vote_tie(ref_tr, l, k):
    """Adjacent alive votes (descending) among the first k+1 that sit within TIE_VOTE of each
    other (relative to the largest |vote|): the order of the elected list is a near-tie."""
    na = int(ref_tr["n_alive"][l])
    if na == 0:
        return False
    v = np.sort(ref_tr["votes"][l][ref_tr["votes"][l] != 0])[::-1]
    if v.size < 2:
        return False
    scale = max(1e-30, float(np.max(np.abs(v))))
    gaps = v[: min(k + 1, v.size) - 1] - v[1: min(k + 1, v.size)]
    return bool(np.any(gaps <= TIE_VOTE * scale))


def compare_trace_ties(gpu_tr, ref_tr, L, b=0):
    """compare_trace, with mismatches the reference's own near-ties explain split off.
    Returns (bad, ties): `ties` lists the layers where k or the elected list differ at an
    election that is a near-tie in the reference (k from n*(1-EMA) within TIE_K of an
    integer, or two votes within TIE_VOTE); `bad` everything else."""
    bad, ties = [], []
    for l, what in compare_trace(gpu_tr, ref_tr, L, b):
        k = int(ref_tr["k"][l])
        if what.startswith("k ") and election_near_tie(ref_tr, l, int(ref_tr["n_alive"][l])):
            ties.append((l, what))
        elif what.startswith("sel ") and _vote_tie(ref_tr, l, k):
            ties.append((l, what))
        elif what == "w" and _vote_tie(ref_tr, l, k):
            ties.append((l, what))
        else:
            bad.append((l, what))
    return bad, ties


def sample_near_tie(ref_logits, gpu_logits, temp, top_k, state):
    """Whether the reference's sample() at this step sits closer to a decision boundary than
    the measured GPU/oracle logit difference can move it (janusdoe.c:3637-3645).

    With d = max|gpu - ref| / temp, every scaled logit moves by at most d, every softmax
    probability by a factor within exp(+-2d), so every cumulative sum by at most ~2d.  The
    draw is a near-tie when r lies within 4d (+1e-6) of the cumulative boundary it fell
    between, or when the k-th and (k+1)-th largest scaled logits are within 2d (the top-k
    threshold could change).  Returns (near_tie, margin)."""
    t = np.float32(temp)
    x = (np.asarray(ref_logits, np.float32) / t).astype(np.float32)
    d = float(np.max(np.abs(np.asarray(gpu_logits, np.float64) - np.asarray(ref_logits, np.float64)))) / float(t)
    V = x.size
    if 0 < top_k < V:
        s = np.sort(x)[::-1]
        if float(s[top_k - 1]) - float(s[top_k]) <= 2 * d + 1e-7:
            return True, 0.0
        x = np.where(x < s[top_k - 1], np.float32(-1e30), x).astype(np.float32)
    e = np.exp((x - np.max(x)).astype(np.float32)).astype(np.float32)
    p = (e / np.float32(np.add.reduce(e, dtype=np.float32))).astype(np.float32)
    cum = np.add.accumulate(p, dtype=np.float32)
    st = int(state)
    st ^= (st << 13) & 0xFFFFFFFFFFFFFFFF
    st ^= st >> 7
    st ^= (st << 17) & 0xFFFFFFFFFFFFFFFF
    r = np.float32(st & 0x7FFFFFFF) / np.float32(0x7FFFFFFF)
    idx = int(np.searchsorted(cum, r, side="left"))
    idx = min(idx, V - 1)
    lo = float(r) - float(cum[idx - 1]) if idx > 0 else float("inf")
    hi = float(cum[idx]) - float(r)
    margin = min(lo, hi)
    return margin <= 4 * d + 1e-6, margin
