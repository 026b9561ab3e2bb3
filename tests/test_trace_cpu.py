"""The decode phase-trace tool's analysis (kore_b200/trace_decode.py) on
synthetic records: launches are split at each return from merge CTAs to
decode CTAs, CTAs that returned early (no end stamp) are left out of the
phases, and the steady-state means skip the first and last launch. CPU only:
the trace build itself runs on a GPU machine."""
import numpy as np

from kore_b200.trace_decode import REC, launches, phase_table


def _rec(kind, t):
    r = np.zeros(1, REC)[0]
    r["kind"] = kind
    r["t"] = t
    return r


def _synthetic(n_launch=5, period=25_000, n_dec=4, n_mer=2):
    recs = []
    for i in range(n_launch):
        b = i * period
        for c in range(n_dec):
            recs.append(_rec(0, [b + 100 * c, b + 1_000, b + 2_000, b + 20_000 + 10 * c, b + 21_000 + 10 * c]))
        recs.append(_rec(0, [b + 500, b + 900, 0, 0, 0]))   # a CTA past its split count: returns early
        for _ in range(n_mer):
            recs.append(_rec(2, [b + 20_000, b + 20_100, b + 21_100, 0, b + 22_000]))
    return np.array(recs, REC)


def test_launches_split_at_merge_to_decode_transitions():
    ls = launches(_synthetic())
    assert len(ls) == 5
    for dec, mer in ls:
        assert len(dec) == 5 and len(mer) == 2
        assert (dec["kind"] == 0).all() and (mer["kind"] == 2).all()


def test_phase_table_means_in_microseconds():
    tab = phase_table(launches(_synthetic()))
    assert tab["launches"] == 5 and tab["steady_launches"] == 3
    m = tab["mean_us"]
    assert abs(m["period"] - 25.0) < 1e-9
    assert abs(m["released"][1] - 1.0) < 1e-9        # the early-returning CTA is not counted
    assert abs(m["tiles"][0] - 20.0) < 1e-9 and abs(m["tiles"][2] - 20.03) < 1e-9
    assert abs(m["merge_seen_last"] - 21.1) < 1e-9 and abs(m["merge_end_last"] - 22.0) < 1e-9
