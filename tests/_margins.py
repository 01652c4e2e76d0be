"""Decision margins of token selection (test infrastructure).

A device token stream may leave the reference's only where the reference's
own decision was a near-tie: where a logit perturbation no larger than the
device's observed logit error could flip the draw. This module measures, for
every draw of a reference run, how far (in raw logit units) the logits would
have to move to change the token sample_next_token picks
(src/cli/sampling.c:38-207):

- greedy: the gap between the largest and the second-largest logit;
- top-k / top-p at temperature T: the smallest of
  - the draw margin: min(r - c[j-1], c[j] - r) / S, where c are the
    cumulative weights of the sorted candidates, S their sum and r = u * S;
    a raw logit error e moves every weight ratio by at most a factor
    exp(2e/T), so the margin converts to logits as m * T / 2;
  - the nucleus cut (top-p): |cumsum/sum_all - p| at the cut and at the
    position before it, converted the same way, counted only when moving
    the cut by one candidate changes the token;
  - the order margin: the raw logit gap between the chosen candidate and its
    sorted neighbours.

Tests accept a divergence at (sequence, draw) only when the reference's
margin there is below 10x the device's observed maximum absolute logit error
(the token-stream rule of the parity contract), and compare the sequence no
further after it.
"""
import numpy as np

GREEDY, TOPK, TOPP = 0, 1, 2


def _stable_desc(x):
    # descending, ties in ascending index order (glibc's merge sort keeps them)
    return np.argsort(-x, kind="stable")


def _weights(xs):
    with np.errstate(invalid="ignore", over="ignore"):
        w = np.exp((xs - xs[0]).astype(np.float64))
    return np.nan_to_num(w, nan=0.0).astype(np.float32)


def _draw(w, n_c, u):
    """Index (into the sorted order) the draw lands on, plus the draw margin
    in probability units."""
    c = np.cumsum(w[:n_c].astype(np.float64))
    S = c[-1]
    r = float(np.float32(u)) * S
    j = int(np.searchsorted(c, r, side="left"))
    j = min(j, n_c - 1)
    lo = c[j - 1] if j > 0 else 0.0
    return j, min(r - lo, c[j] - r) / S


def _nucleus(w, p):
    tot = np.cumsum(w.astype(np.float64))
    norm = tot / tot[-1]
    n_c = int(np.searchsorted(norm, p, side="left")) + 1
    return min(max(n_c, 1), len(w)), norm


def draw_margin(logits, token, strategy, temperature=0.0, top_k=0, top_p=0.0, u=None):
    """Margin (raw logit units) of one draw taken from `logits` (already
    masked, before temperature) that chose `token`. 0 when the float64
    restatement here disagrees with the recorded token (a tie by definition)."""
    x = np.asarray(logits, np.float32)
    if strategy == GREEDY or temperature <= 0.0 or u is None:
        order = _stable_desc(x)
        if int(order[0]) != int(token):
            return 0.0
        return float(x[order[0]]) - float(x[order[1]])
    T = float(temperature)
    with np.errstate(over="ignore"):   # -FLT_MAX / T is -inf, as in the reference
        xs_all = (x * np.float32(1.0 / np.float32(temperature))).astype(np.float32)
    order = _stable_desc(xs_all)
    xs = xs_all[order]
    raw = x[order].astype(np.float64)
    w = _weights(xs)
    if strategy == TOPK:
        n_c = min(int(top_k), len(x))
        norm = None
    else:
        n_c, norm = _nucleus(w, top_p)
    j, dm = _draw(w, n_c, u)
    if int(order[j]) != int(token):
        return 0.0
    margins = [dm * T / 2.0]
    if norm is not None:
        # moving the nucleus cut by one candidate
        for alt in (n_c - 1, n_c + 1):
            if 1 <= alt <= len(x):
                ja, _ = _draw(w, alt, u)
                if int(order[ja]) != int(token):
                    edge = min(n_c - 1 if alt < n_c else n_c, len(x) - 1)
                    margins.append(abs(norm[edge] - top_p) * T / 2.0)
    # swapping the chosen candidate with a sorted neighbour
    for nb in (j - 1, j + 1):
        if 0 <= nb < len(x):
            margins.append(abs(raw[j] - raw[nb]))
    return float(min(margins))


def stream_margins(logits, tokens, strategy, temperature=0.0, top_k=0, top_p=0.0, units=None):
    """logits [n_seq, n_new, V], tokens [n_seq, n_new], units [n_seq, n_new]
    (the unit draw of each sampled token) -> margins [n_seq, n_new]."""
    n_seq, n_new = tokens.shape
    out = np.zeros((n_seq, n_new), np.float32)
    for q in range(n_seq):
        for i in range(n_new):
            out[q, i] = draw_margin(logits[q, i], tokens[q, i], strategy, temperature, top_k, top_p,
                                    None if units is None else units[q, i])
    return out


def unit_draws(rng_stream, rng_unit, seeds, n_new, stream_id):
    """The unit draw consumed by each sampled token of each sequence: one
    dranzer_rng_unit per draw from dranzer_rng_stream(seed, SAMPLING)."""
    out = np.zeros((len(seeds), n_new), np.float64)
    for q, s in enumerate(seeds):
        st = np.array([rng_stream(int(s), stream_id)], np.uint64)
        for i in range(n_new):
            out[q, i] = rng_unit(st)
    return out


def first_divergences(got, ref):
    """(sequence, draw) of the first token where `got` leaves `ref`."""
    bad = []
    for q in range(ref.shape[0]):
        diff = np.nonzero(got[q] != ref[q])[0]
        if diff.size:
            bad.append((q, int(diff[0])))
    return bad


def check_streams(got, ref, margins, logit_err, factor=10.0):
    """Identical streams, or first divergences only where the reference's own
    margin is below factor x the observed maximum absolute logit error.
    Returns the list of accepted divergences; raises AssertionError listing
    any divergence at a decision the error cannot explain."""
    bad = first_divergences(got, ref)
    unexplained = [(q, i, float(margins[q, i])) for q, i in bad if not margins[q, i] < factor * logit_err]
    assert not unexplained, (f"token divergences at decisions with margins above {factor} x the observed "
                             f"logit error {logit_err:.3g}: {unexplained}")
    return bad
