"""vvli_b200.trace.summarize on a synthetic megakernel timeline (no GPU)."""

import numpy as np

from vvli_b200 import trace as T


def timeline(n_layers, grid, spans):
    """Stamps in ns: every CTA starts a phase at the previous release, loads for
    1 us, works for `main` us, writes for 0.5 us; CTA c arrives c ns later than
    CTA 0 (spread), the release comes 1.2 us after the last arrival."""
    names = T.phase_names(2 + 5 * n_layers, n_layers)
    t = np.zeros((len(names), grid, 6), dtype=np.uint64)
    now = 1_000_000
    for f, name in enumerate(names):
        main = spans.get(name.split("_")[0], 2.0)
        for c in range(grid):
            st = now
            inp = st + 1000
            cons = inp + int(main * 1000)
            outw = cons + 500 + c
            t[f, c, :5] = [st, inp, cons, outw, 0]
        release = int(t[f, :, 3].max()) + 1200
        t[f, :, 4] = release
        t[f, :, 5] = now
        now = release
    return t.reshape(-1)


def test_phase_names_layout():
    names = T.phase_names(2 + 5 * 3, 3)
    assert names[0] == "embed" and names[-1] == "lm_head"
    assert names[1:6] == list(T.KINDS) and len(names) == 17
    assert T.phase_names(5, 3) == [f"phase{i}" for i in range(5)]


def test_summarize_figures():
    grid = 8
    raw = timeline(2, grid, {"gu": 10.0, "qkv": 3.0})
    out = T.summarize(raw, grid, 2)
    gu = out["gu"]
    tol = 0.006  # figures are rounded to 0.01 us
    assert abs(gu["prologue"] - 1.0) < tol
    assert abs(gu["main"] - 10.0) < tol
    assert abs(gu["epilogue"] - 0.5035) < tol  # median CTA: 0.5 us + 3.5 ns
    assert abs(gu["barrier"] - 1.2) < tol
    assert abs(gu["spread"] - 0.0035) < tol   # last arrival 7 ns after CTA 0, median 3.5 ns
    # span = release to release: load + main + write + the slowest CTA + barrier
    assert abs(gu["span"] - (1.0 + 10.0 + 0.5 + 0.007 + 1.2)) < tol
    assert abs(out["qkv"]["main"] - 3.0) < tol
    per_layer = sum(out[k]["span"] for k in T.KINDS)
    assert abs(out["per_layer_us"] - round(per_layer, 1)) < 1e-9


def test_stale_stamps_are_ignored():
    # a CTA without an attention item keeps older [1]/[2] stamps: they must not count
    grid = 4
    raw = timeline(1, grid, {}).reshape(-1, grid, 6)
    attn = 2
    raw[attn, 3, 1] = 5  # earlier than this step's start
    raw[attn, 3, 2] = 6
    out = T.summarize(raw.reshape(-1), grid, 1)
    assert abs(out["attn"]["prologue"] - 1.0) < 0.006 and abs(out["attn"]["main"] - 2.0) < 0.006
