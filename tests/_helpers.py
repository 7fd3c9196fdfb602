"""Shared checks of the parity tests: the tolerances of the benchmark's north star, written once.

* Detection masks: bit-exact except pixels whose oracle page-level probability lies within
  MASK_BAND of the threshold.
* Recognition: identical arg-max class at every time step, except steps where the class the
  GPU chose is, in the oracle's own logits, within ARGMAX_TIE of the oracle's maximum (a tie
  at the oracle's precision); per-step softmax probabilities within PROB_TOL absolute.
"""
import numpy as np

MASK_BAND = 1e-3
PROB_TOL = 1e-3
ARGMAX_TIE = 1e-4


def mask_parity(bits_gpu, bits_ref, prob_ref, thr, w):
    """Returns (number of differing pixels outside the band, pixels inside the band)."""
    h = bits_ref.shape[0]
    x = np.arange(w)
    gb = (bits_gpu[:, x // 32] >> (x % 32).astype(np.uint32)) & 1
    rb = (bits_ref[:, x // 32] >> (x % 32).astype(np.uint32)) & 1
    band = np.abs(prob_ref - thr) < MASK_BAND
    bad = (gb != rb) & ~band
    # bits past the page width in the last word must be zero
    tail = 32 * bits_gpu.shape[1] - w
    if tail:
        extra = bits_gpu[:, -1] >> np.uint32(32 - tail)
        assert (extra == 0).all(), "bits past the page width are set"
    return int(bad.sum()), int(band.sum())


def argmax_parity(best_gpu, logits_ref):
    """best_gpu [rows], logits_ref [rows, classes]: number of rows whose GPU class is not the
    oracle's maximum nor within ARGMAX_TIE of it, and the number of such near-tie rows."""
    rows = np.arange(len(best_gpu))
    top = logits_ref.max(axis=1)
    at = logits_ref[rows, best_gpu.astype(np.int64)]
    exact = best_gpu == logits_ref.argmax(axis=1)
    tie_ok = (~exact) & (top - at <= ARGMAX_TIE)
    bad = (~exact) & ~tie_ok
    return int(bad.sum()), int(tie_ok.sum())


def softmax(x):
    m = x.max(axis=-1, keepdims=True)
    e = np.exp(x - m)
    return e / e.sum(axis=-1, keepdims=True)
