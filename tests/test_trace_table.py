"""The per-phase table of c2slm_b200.trace on a synthetic trace (no GPU)."""
import numpy as np

from c2slm_b200.trace import phase_table


def test_phase_table_critical_path_and_medians():
    S, L, G = 2, 2, 3
    NP = 1 + 5 * L
    tr = np.zeros((S, NP, G, 8), np.int64)
    t = 0
    for s in range(S):
        for p in range(NP):
            for c in range(G):
                tr[s, p, c, 0] = t + 100 * c           # starts skewed by CTA
                tr[s, p, c, 1] = t + 100 * c + 500     # prologue 500 ns
                tr[s, p, c, 3] = t + 100 * c + 2000    # busy 2 us
            t += 3000
    out = phase_table(tr)
    # every phase ends 3 us after the previous phase's last end (the logits
    # phase, first of a step, is measured from its own first start)
    assert out["qkv"]["crit_us"] == 3.0 and out["down"]["crit_us"] == 3.0
    assert out["logits"]["crit_us"] == 2.2
    assert out["gateup"]["busy_med_us"] == 2.0 and out["gateup"]["prologue_med_us"] == 0.5
    assert "prologue_med_us" not in out["attn"]
