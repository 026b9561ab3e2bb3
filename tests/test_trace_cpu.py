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


def _prod(kind, tag, cols, out_mode, n_seg, t):
    r = _rec(kind, t)
    r["tag"] = tag
    r["pad2"] = cols | out_mode << 32 | n_seg << 40
    return r


def test_step_launches_order_products_and_decodes_by_start():
    from kore_b200.trace_decode import step_launches, step_table
    E, FF = 3584, 18944
    recs, prods = [], []
    period = 100_000
    for i in range(4):   # four layers: qkv, attention (+ merge), wo, gate/up, down
        b = i * period
        for c in range(3):
            prods.append(_prod(3, E, E, 0, 3, [b + c, b + 2_000, b + 4_000, b + 5_000, b + 9_000 + c]))
        for c in range(3):
            recs.append(_rec(0, [b + 10_000 + c, b + 12_000, b + 13_000, b + 38_000, b + 39_000]))
        recs.append(_rec(2, [b + 38_500, b + 38_600, b + 39_100, 0, b + 40_000]))
        for c in range(3):
            prods.append(_prod(3, E, E, 1, 1, [b + 41_000 + c, b + 43_000, b + 44_000, b + 45_000, b + 50_000]))
        for c in range(3):
            prods.append(_prod(4, FF, E, 2, 2, [b + 51_000 + c, b + 53_000, b + 54_000, b + 55_000, b + 80_000]))
        for c in range(3):
            prods.append(_prod(3, E, FF, 1, 1, [b + 81_000 + c, b + 83_000, b + 84_000, b + 85_000, b + 99_000]))
    ls = step_launches(np.array(recs + prods, REC), E)
    assert [l["role"] for l in ls[:5]] == ["qkv", "attn", "wo", "gate_up", "down"]
    assert len(ls) == 20
    tab = step_table(ls)
    m = tab["mean_us"]
    assert abs(m["attn"]["end_last"] - 30.0) < 1e-9        # the merge CTA's end counts
    assert abs(m["qkv"]["landed_med"] - 5.0) < 1e-9
    assert abs(m["wo"]["gap_from_prev_end"] - 3.0) < 1e-9   # 40 us merge end -> 43 us release
    assert abs(m["gate_up"]["period"] - 30.0) < 1e-9
