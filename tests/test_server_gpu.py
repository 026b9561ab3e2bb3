"""Many chat sessions over one context (kore_cuda_server_*) against kore's own
chat flow, through the C ABI.

kore serves one conversation at a time: prefill() appends a turn with
forward_batch, gen_step() samples greedily, appends and runs forward()
(kore.cpp:1720-1756); condense() rebuilds the cache from position 0
(kore.cpp:1786-1797). The reference here is exactly that flow run by kore
itself (oracle/engine_harness.cpp, keng_turn_ref), one session at a time.
The server runs several sessions at once over the shared page pool, the
whole model on the device, their decode steps queued back to back each
round; every session's tokens must equal kore's for its own conversation,
across turns, a condense and a session closed and reopened.
"""
import numpy as np
import pytest

import kore_b200 as K
import oracle.oracle as O
from tests.test_step_gpu import engine_model

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not O.engine_available(), reason="oracle/_ref/libkore_engine.so not built")]

L, E, H, G, FF, V, CTX = 2, 1024, 8, 2, 1280, 96, 512


def make_server(eng, max_seqs):
    g = K.KoreCuda(L, H, G, E // H, CTX, max_seqs=max_seqs)
    m = engine_model(eng, L)
    g.set_model(FF, V, O.engine_lib().keng_rms_eps(eng.h), m["tok_embd"], m["out_norm"], m["out_w"], m["layers"])
    return g, K.Server(g, eos=V, bos=V + 1)   # ids the vocabulary never produces: turns end at max_new


def run_until_idle(srv, sessions):
    got = {s: [] for s in sessions}
    for _ in range(1000):
        ev = srv.step()
        if not ev:
            return got
        for s, tok, st in ev:
            assert st in (K.EV_TOKEN, K.EV_LIMIT), (s, tok, st)
            got[s].append(tok)
    raise AssertionError("sessions never went idle")


def test_sessions_match_kores_chat_flow():
    eng = O.GreedyEngine(L, E, H, G, FF, V, ctx=CTX, seed=404, threads=4)
    g, srv = make_server(eng, max_seqs=4)
    rng = np.random.default_rng(405)
    prompts = [rng.integers(0, V, n).tolist() for n in (70, 40, 130)]
    n_new = [12, 20, 6]
    sess = [srv.open() for _ in prompts]
    for s, p, n in zip(sess, prompts, n_new):
        srv.submit(s, p, max_new=n)
    got = run_until_idle(srv, sess)
    for s, p, n in zip(sess, prompts, n_new):
        assert got[s] == eng.turn_ref(p, 0, n), f"session {s}, first turn"
        assert srv.history(s) == p + got[s]

    # a second turn for session 0 while session 2 also continues
    t0, t2 = rng.integers(0, V, 25).tolist(), rng.integers(0, V, 9).tolist()
    srv.submit(sess[0], t0, max_new=8)
    srv.submit(sess[2], t2, max_new=15)
    got2 = run_until_idle(srv, [sess[0], sess[2]])
    for s, p, n, t, n2 in ((sess[0], prompts[0], n_new[0], t0, 8), (sess[2], prompts[2], n_new[2], t2, 15)):
        first = eng.turn_ref(p, 0, n)                 # kore replays the session's first turn
        assert got2[s] == eng.turn_ref(t, len(p) + n, n2), f"session {s}, second turn"
        assert first == got[s]

    # condense session 1: its cache rebuilt from position 0 over a shorter
    # history, then a new turn
    hist = srv.history(sess[1])
    new_hist = rng.integers(0, V, 12).tolist() + hist[-30:]
    srv.condense(sess[1], new_hist)
    t1 = rng.integers(0, V, 7).tolist()
    srv.submit(sess[1], t1, max_new=10)
    got3 = run_until_idle(srv, [sess[1]])
    eng.turn_ref(new_hist, 0, 0)
    assert got3[sess[1]] == eng.turn_ref(t1, len(new_hist), 10), "after condense"

    # a session closed and reopened starts empty and reuses the pool
    srv.close_session(sess[2])
    s_new = srv.open()
    p = rng.integers(0, V, 33).tolist()
    srv.submit(s_new, p, max_new=5)
    assert run_until_idle(srv, [s_new])[s_new] == eng.turn_ref(p, 0, 5)
    srv.close()
    g.close()


def test_server_errors():
    eng = O.GreedyEngine(L, E, H, G, FF, V, ctx=CTX, seed=406, threads=2)
    g, srv = make_server(eng, max_seqs=2)
    a, b = srv.open(), srv.open()
    with pytest.raises(K.KoreCudaError) as e:
        srv.open()                                   # every slot taken
    assert e.value.code == -3
    with pytest.raises(K.KoreCudaError) as e:
        srv.submit(a, [1] * CTX)                     # kore's prefill(): no room in the context
    assert e.value.code == -2
    with pytest.raises(K.KoreCudaError) as e:
        srv.submit(a, [V + 3])                       # outside the vocabulary
    assert e.value.code == -2
    srv.close_session(b)
    with pytest.raises(K.KoreCudaError) as e:
        srv.submit(b, [1, 2])                        # closed
    assert e.value.code == -2
    srv.submit(a, [1, 2, 3], max_new=2)
    assert [t for _, t, _ in srv.step()] == eng.turn_ref([1, 2, 3], 0, 1)
    srv.close()
    g.close()
