"""Parity helpers shared by the GPU tests, the smoke check and bench.py.

Rules: encoder output and joint values within max relative error 1e-3 of
the oracle per chunk, rel = max|d| / max|ref| (the definition of the reference's
tools/compare.py:30); emitted token ids identical wherever the oracle's top-2 joint margin
exceeds 1e-3 (a near-tie may flip and is logged, not failed).
"""
import numpy as np

REL_TOL = 1e-3
MARGIN = 1e-3


def rel_err(got, ref):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    if ref.size == 0:
        return 0.0
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


def per_chunk_rel(got, ref, chunk_rows):
    out, r0 = [], 0
    for c in chunk_rows:
        out.append(rel_err(got[r0:r0 + c], ref[r0:r0 + c]))
        r0 += c
    return out


def tokens_match(got, ref_tokens, dec_token=None, dec_margin=None, blank=None):
    """Returns (ok, note). When the sequences differ, the first difference is accepted only if
    one of the oracle's decisions leading to it had a top-2 margin below MARGIN."""
    got, ref_tokens = list(got), list(ref_tokens)
    if got == ref_tokens:
        return True, "identical"
    k = next((i for i, (a, b) in enumerate(zip(got, ref_tokens)) if a != b), min(len(got), len(ref_tokens)))
    if dec_token is None:
        return False, f"tokens differ at {k}"
    # decisions of the oracle between emitted token k-1 and emitted token k (inclusive); when the
    # token inserted or dropped at k repeats the tokens just before it, the flipped decision may sit
    # anywhere in that run of equal tokens, so the window starts where the run starts
    emitted = np.nonzero(np.asarray(dec_token) != blank)[0]
    moved = {t for t in (got[k] if k < len(got) else None, ref_tokens[k] if k < len(ref_tokens) else None) if t is not None}
    s0 = k
    while s0 >= 1 and ref_tokens[s0 - 1] in moved:
        s0 -= 1
    lo = emitted[s0 - 1] + 1 if s0 >= 1 and s0 - 1 < len(emitted) else 0
    hi = emitted[k] + 1 if k < len(emitted) else len(dec_token)
    window = np.asarray(dec_margin)[lo:hi]
    if window.size and window.min() < MARGIN:
        return True, f"near-tie at token {k} (oracle margin {window.min():.2e})"
    return False, f"tokens differ at {k} (oracle margins >= {window.min() if window.size else float('nan'):.2e})"
