"""Phase timeline of one decode-megakernel step (contexts created with VVLI_TRACE=1).

vvli_cuda_trace returns, per phase f and CTA c, six %globaltimer stamps:
[0] consumers start the phase, [1] inputs loaded, [2] rows consumed,
[3] outputs written (the CTA arrives at the grid barrier), [4] barrier
passed, [5] producer issued the phase's first weight stage.  In attention
phases [1] is "q and page numbers loaded", [5] "first page's scores done",
[2] "pages done" and [3] includes the merge of the split partials.

summarize() reduces one step to microseconds per phase kind, averaged over
layers: the phase's span (barrier release to barrier release), the median
CTA's prologue / main part / epilogue, the barrier's latency (last arrival
to release) and its spread (median arrival to last arrival, the imbalance).
"""

from __future__ import annotations

import numpy as np

KINDS = ("qkv", "attn", "o", "gu", "down")


def phase_names(n_phases: int, n_layers: int) -> list:
    if n_phases == 2 + len(KINDS) * n_layers:
        return ["embed"] + [k for _ in range(n_layers) for k in KINDS] + ["lm_head"]
    return [f"phase{i}" for i in range(n_phases)]


def _median(v: np.ndarray) -> float:
    return float(np.median(v)) if v.size else 0.0


def summarize(raw, grid: int, n_layers: int) -> dict:
    """Per phase kind: mean over layers of the figures above, in microseconds."""
    t = np.asarray(raw, dtype=np.int64).reshape(-1, grid, 6)
    names = phase_names(t.shape[0], n_layers)
    rows = {}
    prev_release = None
    for f, name in enumerate(names):
        st, inp, cons, outw, rel = (t[f, :, k] for k in range(5))
        live = st > 0
        release = int(rel[live].max()) if live.any() else 0
        begin = prev_release if prev_release is not None else int(st[live].min()) if live.any() else 0
        has_in = live & (inp >= st)  # stamps of this step only (a CTA without an item keeps older ones)
        has_c = has_in & (cons >= inp)
        arrive = outw[live & (outw > 0)]
        fig = {
            "span": (release - begin) / 1e3,
            "prologue": _median((inp - st)[has_in]) / 1e3,
            "main": _median((cons - inp)[has_c]) / 1e3,
            "epilogue": _median((outw - cons)[has_c & (outw > 0)]) / 1e3,
            "barrier": (release - int(arrive.max())) / 1e3 if arrive.size else 0.0,
            "spread": (int(arrive.max()) - _median(arrive)) / 1e3 if arrive.size else 0.0,
        }
        rows.setdefault(name, []).append(fig)
        prev_release = release
    out = {}
    for name, figs in rows.items():
        out[name] = {k: round(float(np.mean([g[k] for g in figs])), 2) for k in figs[0]}
    layer = sum(out[k]["span"] for k in KINDS if k in out)
    out["per_layer_us"] = round(layer, 1)
    return out
