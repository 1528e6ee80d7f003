"""Test infrastructure (the checker, not the product): restatement of the reference's
semantic-code sampler, used to check the engine's device sampler (k_fm_sample /
vx_selftest_top_p) index for index.

sample_top_p follows sampleTopP, src/engine.ts:247-289, step by step with the number
types of its JavaScript:
- `scaled` is a Float32Array, so logits[i] / temperature (a double division) is
  rounded to f32 when stored (:251-252);
- the maximum is taken over those f32 values (:255-256);
- exp(scaled[i] - maxV) is a double, rounded to f32 when stored back, and sumExp adds
  the stored f32 values sequentially in double (:257-261);
- the probabilities are f32(scaled[i] / sumExp) (:262);
- Array.prototype.sort is stable, so equal probabilities keep index order (:265-266);
- the running sum is a sequential double sum over the sorted probabilities; the cutoff
  is one past the first position whose sum reaches top_p, else n (:269-277); the
  renormalising sum repeats the same additions, so it equals the running sum at the
  cutoff (:280-281);
- r = u * reSum with u the caller's draw in place of Math.random(); the result is the
  first index (in sorted order, before the cutoff) whose running sum reaches r, else
  the top index (:282-288).
The masking of generate() (index 0 and >= 8194 set to -Infinity, :2559-2563) is the
caller's: mask_semantic() restates it.
"""
import numpy as np

VALID_SEMANTIC = 8194


def mask_semantic(logits) -> np.ndarray:
    lg = np.array(logits, dtype=np.float32, copy=True)
    lg[0] = -np.inf
    lg[VALID_SEMANTIC:] = -np.inf
    return lg


def sample_top_p(logits, top_p: float, temperature: float, u: float, return_margin: bool = False):
    """Index chosen by sampleTopP for the draw u.  With return_margin, also the smallest
    distance between a running sum that decided the result and its threshold (the
    device adds in a tree, not sequentially; a margin above ~1e-12 means the order of
    the additions cannot change the result)."""
    lg = np.asarray(logits, dtype=np.float32)
    n = lg.size
    scaled = (lg.astype(np.float64) / temperature).astype(np.float32)
    max_v = scaled.max()
    with np.errstate(invalid="ignore"):
        e = np.exp(scaled.astype(np.float64) - np.float64(max_v)).astype(np.float32)
    sum_exp = np.add.accumulate(e.astype(np.float64))[-1]
    p = (e.astype(np.float64) / sum_exp).astype(np.float32)
    order = np.argsort(-p, kind="stable")
    cum = np.add.accumulate(p[order].astype(np.float64))
    hit = np.nonzero(cum >= top_p)[0]
    cutoff = int(hit[0]) + 1 if hit.size else n
    re_sum = cum[cutoff - 1]
    r = u * re_sum
    walk = np.nonzero(cum[:cutoff] >= r)[0]
    pick = int(walk[0]) if walk.size else 0
    idx = int(order[pick])
    if not return_margin:
        return idx
    # the comparisons that decided the result: the sum that reached top_p and the one
    # before it (or the total, when none did); the sum before the pick (it fell short
    # of r) and the pick's own unless it already equals the renormalising sum (only
    # zeros follow it; u < 1 keeps r at or below that sum in any order of additions)
    if hit.size:
        margins = [abs(cum[cutoff - 1] - top_p)] + ([abs(cum[cutoff - 2] - top_p)] if cutoff >= 2 else [])
    else:
        margins = [abs(cum[-1] - top_p)]
    if pick >= 1:
        margins.append(abs(cum[pick - 1] - r))
    if walk.size and cum[pick] < re_sum:
        margins.append(abs(cum[pick] - r))
    return idx, min(margins)
