"""Worker of tests/test_multigpu.py (one process per GPU, launched by
torch.distributed.run): a KV-sharded context per GPU, handles exchanged over
gloo, decode steps through kore_cuda_attn_decode_sharded_dev compared with
the oracle on every rank, then the attention block with its projections on
the same split (kore_cuda_attn_block_decode_dev): identical on every rank,
its projections bit-exact and its attention within tolerance of the oracle;
a prefill chunk on the split merged through the exchange; and the whole
model on the split (device prefill, then decode steps): greedy IDs equal to
kore's own on every rank."""
import datetime
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import kore_b200 as K  # noqa: E402
from kore_b200.shard import exchange_handles  # noqa: E402
from oracle import oracle as O  # noqa: E402
from tests.attn_check import assert_attn_close, normal  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    H, G, d, ctx_max, cached = 28, 4, 128, 4096, 3000   # 3000 + 5 + 200 + 1 positions used
    ctx = K.KoreCuda(2, H, G, d, ctx_max, device=local, shard_rank=rank, shard_count=world)
    oras = [O.OracleLayer(H, G, d, ctx_max) for _ in range(2)]
    for layer in range(2):
        k, v = normal(500 + layer, (cached, G * d), (cached, G * d))
        ctx.append(0, layer, 0, k, v)
        oras[layer].fill(0, k, v)
    exchange_handles(ctx, dist)
    dev = torch.device("cuda", local)
    out = torch.empty(H * d, device=dev)
    for step in range(3):
        for layer in range(2):
            pos = cached + step
            q, k, v = normal(600 + 10 * step + layer, (H * d,), (G * d,), (G * d,))
            tq, tk, tv = (torch.from_numpy(x).to(dev) for x in (q, k, v))
            torch.cuda.synchronize()
            ctx.decode_sharded_dev(0, layer, pos, tq, tk, tv, out)
            ctx.sync()
            assert_attn_close(out.cpu().numpy().reshape(H, d), oras[layer].decode(pos, q, k, v),
                              f"rank {rank} step {step} layer {layer}")
    # the attention block on the split: every rank computes the projections
    from kore_b200.qweights import Q4_K, Q6_K, random_qmat
    E, kvd = H * d, G * d
    rng = np.random.default_rng(700)   # the same weights on every rank
    mats, biases = [], []
    for layer in range(2):
        m = [random_qmat(t, r, E, rng) for t, r in ((Q4_K, E), (Q4_K, kvd), (Q6_K, kvd), (Q4_K, E))]
        b = [rng.standard_normal(n).astype(np.float32) for n in (E, kvd, kvd)]
        ctx.set_attn_weights(layer, *m, *b)
        mats.append(m)
        biases.append(b)
    o_dev = torch.empty(E, device=dev)
    for step in range(2):
        for layer in range(2):
            pos = cached + 3 + step
            xb = normal(800 + 10 * step + layer, (E,))[0]
            txb = torch.from_numpy(xb).to(dev)
            torch.cuda.synchronize()
            ctx.attn_block_decode_dev(0, layer, pos, txb, o_dev)
            ctx.sync()
            got = o_dev.cpu().numpy()
            everyone = [None] * world
            dist.all_gather_object(everyone, got.view(np.uint32).tobytes())
            assert all(e == everyone[0] for e in everyone), f"step {step} layer {layer}: ranks disagree"
            m, (bq, bk, bv) = mats[layer], biases[layer]
            rq, rk, rv = O.qmatvec(m[0], xb, bq), O.qmatvec(m[1], xb, bk), O.qmatvec(m[2], xb, bv)
            ratt = oras[layer].decode(pos, rq, rk, rv)
            ref = O.qmatvec(m[3], ratt.reshape(-1))
            err = float(np.abs(got.astype(np.float64) - ref).max())
            assert err <= 2e-2 * max(1.0, float(np.abs(ref).max())), (rank, step, layer, err)
    # a prefill chunk on the split (200 rows, across a page edge), merged over
    # the peer exchange in pieces of 64 queries, then a decode after it
    pos0 = cached + 5
    for layer in range(2):
        q, k, v = normal(900 + layer, (200, H * d), (200, G * d), (200, G * d))
        torch.cuda.synchronize()
        got = ctx.prefill(0, layer, pos0, q, k, v)
        assert_attn_close(got, oras[layer].prefill(pos0, q, k, v), f"rank {rank} prefill layer {layer}")
        q1, k1, v1 = normal(950 + layer, (H * d,), (G * d,), (G * d,))
        got1 = ctx.decode_sharded(0, layer, pos0 + 200, q1, k1, v1)
        assert_attn_close(got1, oras[layer].decode(pos0 + 200, q1, k1, v1), f"rank {rank} decode after prefill")
    dist.barrier()
    ctx.close()

    # the whole model on the split: kore's own random-init model (every rank
    # builds the same one), its prompt prefilled on the device over the
    # split, then decode steps; greedy IDs equal kore's own flow on every rank
    if O.engine_available():
        from tests.test_step_gpu import engine_model
        L, E, Hm, Gm, FF, V, n_prompt, n_gen = 2, 1024, 8, 2, 1280, 96, 300, 12
        eng = O.GreedyEngine(L, E, Hm, Gm, FF, V, ctx=n_prompt + n_gen + 8, seed=77, threads=2)
        prompt = np.random.default_rng(78).integers(0, V, n_prompt)
        ref, _ = eng.generate_ref(prompt, n_gen)
        m = engine_model(eng, L)
        cm = K.KoreCuda(L, Hm, Gm, E // Hm, n_prompt + n_gen + 8, device=local, shard_rank=rank, shard_count=world)
        cm.set_model(FF, V, O.engine_lib().keng_rms_eps(eng.h), m["tok_embd"], m["out_norm"], m["out_w"], m["layers"])
        exchange_handles(cm, dist)
        ids = [cm.prefill_tokens(0, prompt, 0)[0]]
        for i in range(1, n_gen):
            ids.append(cm.decode_step(0, ids[-1], n_prompt + i - 1)[0])
        assert ids == ref.tolist(), (rank, ids, ref.tolist())
        dist.barrier()
        cm.close()
    dist.destroy_process_group()
    print(f"rank {rank} ok", flush=True)


if __name__ == "__main__":
    main()
