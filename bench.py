"""bench.py — decode attention throughput of the B200 kore path.

Workload (the metric's "@7B ctx 32k"): Qwen2.5-7B-shaped
attention, 28 layers, 28 query / 4 KV heads, head_dim 128, one sequence,
fp32 KV cache of 32768 seeded N(0,1) rows per layer (3.5 GiB, far larger than
the 126 MB L2, so no L2 flush is needed between steps). One step = one decode
token through all 28 layers: RoPE of q/k at position 32768, append of k/v,
attention over positions 0..32768.

  value  device-resident: q/k/v already in HBM, CUDA events on the context's
         stream around K replays of a CUDA graph holding one step; max over
         ranks; GB/s of algorithmic bytes
         (per layer: 2*(pos+1)*512*4 K/V + 2*28*128*4 q/out + 2*512*4 append).
  e2e    the same steps through the host-buffer C entry point
         kore_cuda_attn_decode (kore's call: host q/k/v in, host out back),
         wall clock, copies included.
At N > 1 the KV positions are split over the GPUs by page (round robin); each
layer's partial outputs and log-sum-exps are pushed to every peer over NVLink
peer memory and merged on every rank (kore_cuda_attn_decode_sharded_dev), one
exchange per layer. The cache is fixed (strong scaling).

``--impl reference`` times kore's own CPU attention (the reference compiled
in place, oracle/_ref) on this host: kore.cpp forward() per layer on its
fp32 cache, layers fanned over the host's cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

H, G, D = 28, 4, 128
L = 28          # layers (--layers overrides, for small profiling cases)
POS = 32768     # decode position (--pos overrides)
CTX = POS + 1
KVD = G * D


def layer_bytes(pos: int) -> int:
    return 2 * (pos + 1) * KVD * 4 + 2 * H * D * 4 + 2 * KVD * 4


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=100)
    ap.add_argument("--layers", type=int, default=28, help="fewer layers: a small case for ncu captures")
    ap.add_argument("--pos", type=int, default=32768, help="decode position (cached rows per layer)")
    ap.add_argument("--prefill-steps", type=int, default=5)
    ap.add_argument("--prefill-layers", type=int, default=28)
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-batched", action="store_true", help="skip the config-5 batched decode line")
    ap.add_argument("--batched-steps", type=int, default=20)
    ap.add_argument("--no-block", action="store_true", help="skip the attention-block (with projections) line")
    ap.add_argument("--block-steps", type=int, default=100)
    ap.add_argument("--block-only", action="store_true", help="measure only the attention block (development)")
    ap.add_argument("--prefill-only", action="store_true", help="measure only the prefill (development)")
    a = ap.parse_args()
    global L, POS, CTX
    L, POS, CTX = a.layers, a.pos, a.pos + 1
    return a


# ---------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[tuple[float, str]] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()
        t0 = time.time()
        while not self.lines and time.time() - t0 < 3:
            time.sleep(0.02)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def stop(self, t_begin: float, t_end: float) -> dict:
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.15)
        self.proc.terminate()
        self.proc.wait()
        rows = [l for (t, l) in self.lines if t_begin - 0.1 <= t <= t_end + 0.15] or [l for _, l in self.lines[-2:]]
        mhz, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            f = [x.strip() for x in r.split(",")]
            try:
                mhz.append(float(f[1]))
                mx = float(f[2])
            except (ValueError, IndexError):
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(mhz)}


# ---------------------------------------------------------------- our arm

def run_ours(args, rank: int, world: int, dist) -> dict | None:
    import torch
    import kore_b200 as K

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    ctx = K.KoreCuda(L, H, G, D, CTX, device=dev.index, shard_rank=rank, shard_count=world)
    # the context runs on a torch-owned stream, so tensors used on it (and by
    # NCCL) outlive nothing they depend on when the context is closed
    stream = torch.cuda.Stream(device=dev)
    ctx.set_stream(stream.cuda_stream)

    # seeded N(0,1) cache: all rows generated on the device per layer; each
    # shard stores the rows of the pages it holds
    gen = torch.Generator(device=dev)
    with torch.cuda.stream(stream):
        for layer in range(L):
            gen.manual_seed(1000 + layer)
            k = torch.randn(POS, KVD, device=dev, generator=gen)
            v = torch.randn(POS, KVD, device=dev, generator=gen)
            ctx.append_dev(0, layer, 0, POS, k, v)
            del k, v
        gen.manual_seed(7)
        q = torch.randn(L, H * D, device=dev, generator=gen)
        kn = torch.randn(L, KVD, device=dev, generator=gen)
        vn = torch.randn(L, KVD, device=dev, generator=gen)
        out = torch.empty(L, H * D, device=dev)
        part = torch.empty(L, ctx.part_floats, device=dev)
    ctx.sync()

    if world > 1:
        from kore_b200.shard import exchange_handles
        exchange_handles(ctx, dist)     # exchange buffers mapped over CUDA IPC

    def step():
        for layer in range(L):
            if world == 1:
                ctx.decode_dev(0, layer, POS, q[layer], kn[layer], vn[layer], out[layer])
            else:
                # partial on this rank's pages, pushed to the peers over NVLink, merged on every rank
                ctx.decode_sharded_dev(0, layer, POS, q[layer], kn[layer], vn[layer], out[layer])

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
    ctx.sync()
    barrier()

    # one decode step of all layers captured once as a CUDA graph: the
    # per-layer launches then cost no host time inside the timed region (the
    # cross-GPU exchange keeps its epochs on the device, so replays stay in step)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    barrier()
    with torch.cuda.stream(stream):
        for _ in range(3):
            graph.replay()
    ctx.sync()
    run = graph.replay

    clocks = ClockSampler(dev.index)
    clocks.start()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    barrier()
    t_begin = time.time()
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(args.steps):
            run()
        e1.record(stream)
    e1.synchronize()
    t_end = time.time()
    ctx.sync()
    barrier()
    clk = clocks.stop(t_begin, t_end)
    ms = e0.elapsed_time(e1)
    del graph

    # isolated per-launch durations (events around every layer's call, which
    # also removes the overlap between consecutive layers)
    n_ev = min(args.steps, 50)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n_ev * L)]
    with torch.cuda.stream(stream):
        for s in range(n_ev):
            for layer in range(L):
                a, b = evs[s * L + layer]
                a.record(stream)
                if world == 1:
                    ctx.decode_dev(0, layer, POS, q[layer], kn[layer], vn[layer], out[layer])
                else:
                    ctx.decode_partial_dev(0, layer, POS, q[layer], kn[layer], vn[layer], part[layer])
                b.record(stream)
    torch.cuda.synchronize(dev)
    iso_ms = sum(a.elapsed_time(b) for a, b in evs) / len(evs)

    # end to end through the host-buffer entry point (kore's own call shape)
    e2e_ms = None
    if world == 1:
        hq, hk, hv = q.cpu().numpy(), kn.cpu().numpy(), vn.cpu().numpy()
        ho = np.empty((L, H * D), np.float32)
        for layer in range(L):
            ho[layer] = ctx.decode(0, layer, POS, hq[layer], hk[layer], hv[layer]).reshape(-1)
        t0 = time.perf_counter()
        for _ in range(args.e2e_steps):
            for layer in range(L):
                ho[layer] = ctx.decode(0, layer, POS, hq[layer], hk[layer], hv[layer]).reshape(-1)
        e2e_ms = (time.perf_counter() - t0) * 1e3 / args.e2e_steps
    else:
        # host buffers per layer: pinned copies in, merged output back
        hq = q.cpu().pin_memory()
        hk, hv = kn.cpu().pin_memory(), vn.cpu().pin_memory()
        ho = torch.empty(L, H * D).pin_memory()
        barrier()
        t0 = time.perf_counter()
        with torch.cuda.stream(stream):
            for _ in range(args.e2e_steps):
                for layer in range(L):
                    q[layer].copy_(hq[layer], non_blocking=True)
                    kn[layer].copy_(hk[layer], non_blocking=True)
                    vn[layer].copy_(hv[layer], non_blocking=True)
                    ctx.decode_sharded_dev(0, layer, POS, q[layer], kn[layer], vn[layer], out[layer])
                    ho[layer].copy_(out[layer], non_blocking=True)
                    stream.synchronize()
        e2e_ms = (time.perf_counter() - t0) * 1e3 / args.e2e_steps

    t = torch.tensor([ms, iso_ms, e2e_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, iso_ms, e2e_ms = t.tolist()
    block = None
    if world == 1 and not args.no_block:
        block = run_block(args, ctx, stream, dev)
    ctx.close()
    if rank != 0:
        return None

    step_bytes = L * layer_bytes(POS)
    ms_step = ms / args.steps
    gbs = step_bytes / (ms_step * 1e-3) / 1e9
    e2e_gbs = step_bytes / (e2e_ms * 1e-3) / 1e9
    peaks = load_peaks()
    launch_bytes = layer_bytes(POS) / world
    layer_ms = ms_step / L          # one layer's decode (+ split merge) inside the timed region
    achieved = launch_bytes / (layer_ms * 1e-3) / 1e9
    line = {
        "metric": "decode attn HBM GB/s @7B ctx 32k (28 layers, 28Q/4KV, d128, fp32 KV)",
        "value": round(gbs, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_step, 5), "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1) q/k/v and KV cache)",
        "config": {"workload": f"cfg4: Qwen2.5-7B-shaped decode at position {POS}, {L} layers, batch 1",
                   "kv_bytes_per_step": step_bytes, "l2": "inputs 3.5 GiB > L2, no flush needed",
                   "kv_split": f"pages round-robin over {world} GPU(s)" if world > 1 else "none"},
        "e2e": {"value": round(e2e_gbs, 1), "unit": "GB/s", "ms_per_step": round(e2e_ms, 4),
                "h2d_bytes_per_step": L * (H * D + 2 * KVD) * 4, "d2h_bytes_per_step": L * H * D * 4},
        "roofline": {"bound": "hbm", "kernel": "attn_decode_kernel<128,7,8,8,3> + split_merge_kernel<128,7>" + (" + peer_exchange_kernel" if world > 1 else ""),
                     "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "peak_source": peaks["source"],
                     "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": load_traffic(),
                     "launch_ms": round(layer_ms, 5), "launch_ms_isolated": round(iso_ms, 5),
                     "algorithmic_bytes_per_launch": int(launch_bytes),
                     "timing": "launch_ms = timed region / (steps x layers), CUDA events on the context stream; "
                               "launch_ms_isolated = events around each layer's call (no inter-layer overlap)"},
        "gpu_launches": args.steps * L * (3 if world > 1 else 2),
        "clocks": clk,
    }
    if not args.no_cpu_baseline and world == 1:
        line["cpu_baseline"] = cpu_baseline_sample()
    if block is not None:
        proj_ms = block.pop("_cpu_proj_ms", None)
        att = line.get("cpu_baseline", {}).get("attention_ms")
        if proj_ms is not None and att is not None:
            per_layer = block["weight_bytes_per_step"] / L + layer_bytes(POS)
            block["cpu_baseline"] = {
                "value": round(per_layer / ((att + proj_ms) * 1e-3) / 1e9, 3), "unit": "GB/s", "cores": 1,
                "kind": "reference",
                "sample": f"1 of 28 layers: kore's attention at pos {POS} ({att:.1f} ms, as cpu_baseline) + "
                          f"kore's quantize_row_q8_K + matvec_mt of Wq, Wk, Wv, Wo on 1 thread "
                          f"(best of 3, {proj_ms:.2f} ms)"}
        line["attn_block"] = block
    if not args.no_prefill and world == 1:
        line["prefill"] = run_prefill(args, torch.device("cuda", 0), peaks)
    return line


def run_block_only(args) -> dict:
    """The attention-block line alone, on a context set up as run_ours sets it up."""
    import torch
    import kore_b200 as K

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    ctx = K.KoreCuda(L, H, G, D, CTX, device=0)
    stream = torch.cuda.Stream(device=dev)
    ctx.set_stream(stream.cuda_stream)
    gen = torch.Generator(device=dev)
    with torch.cuda.stream(stream):
        for layer in range(L):
            gen.manual_seed(1000 + layer)
            k = torch.randn(POS, KVD, device=dev, generator=gen)
            v = torch.randn(POS, KVD, device=dev, generator=gen)
            ctx.append_dev(0, layer, 0, POS, k, v)
            del k, v
    ctx.sync()
    try:
        d = run_block(args, ctx, stream, dev)
        d.pop("_cpu_proj_ms", None)
        return d
    finally:
        ctx.close()


def run_block(args, ctx, stream, dev) -> dict:
    """The attention block of each layer with its quantised projections on the
    GPU (kore_cuda_attn_block_decode): Q8_K quantisation of the normed input,
    Wq/Wk/Wv products + biases, the config-4 attention at POS, Wo. Seeded
    synthetic GGUF weights in kore's Q4_K_M mix for these tensors (Q4_K; Q6_K
    for Wv), one set per layer, so each step streams every layer's weights
    and KV from HBM."""
    import torch
    import kore_b200 as K
    from kore_b200.qweights import Q4_K, Q6_K, random_qmat

    E = H * D
    rng = np.random.default_rng(77)
    w_bytes = 0
    mats0 = None
    for layer in range(L):
        mats = [random_qmat(t, r, E, rng) for t, r in ((Q4_K, E), (Q4_K, KVD), (Q6_K, KVD), (Q4_K, E))]
        w_bytes += sum(m.nbytes for m in mats)
        b = [rng.standard_normal(n).astype(np.float32) for n in (E, KVD, KVD)]
        ctx.set_attn_weights(layer, *mats, *b)
        if mats0 is None:
            mats0 = mats
    gen = torch.Generator(device=dev)
    gen.manual_seed(78)
    with torch.cuda.stream(stream):
        xb = torch.randn(L, E, device=dev, generator=gen)
        o = torch.empty(L, E, device=dev)

    def step():
        for layer in range(L):
            ctx.attn_block_decode_dev(0, layer, POS, xb[layer], o[layer])

    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            step()
    ctx.sync()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    with torch.cuda.stream(stream):
        for _ in range(3):
            graph.replay()
    ctx.sync()
    steps = args.block_steps
    clocks = ClockSampler(dev.index)
    clocks.start()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    t_begin = time.time()
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(steps):
            graph.replay()
        e1.record(stream)
    e1.synchronize()
    t_end = time.time()
    ctx.sync()
    clk = clocks.stop(t_begin, t_end)
    ms = e0.elapsed_time(e1) / steps
    del graph
    # end to end through the host-buffer entry point (xb in, Wo*att out per layer)
    hx = xb.cpu().numpy()
    for layer in range(L):
        ctx.attn_block_decode(0, layer, POS, hx[layer])
    n_e2e = max(1, args.e2e_steps // 4)
    t0 = time.perf_counter()
    for _ in range(n_e2e):
        for layer in range(L):
            ctx.attn_block_decode(0, layer, POS, hx[layer])
    e2e_ms = (time.perf_counter() - t0) * 1e3 / n_e2e
    # CPU leg: kore's own quantize + matvec_mt of one layer's four matrices on
    # one core (the compiled reference), added to its one-core attention time
    # by the caller
    cpu_proj_ms = None
    if not args.no_cpu_baseline:
        from oracle import oracle as O
        if O.ref_available():
            x = np.random.default_rng(79).standard_normal(E).astype(np.float32)
            cpu_proj_ms = sum(O.ref_qmatvec_ms(m, x, 1, 3)[0] for m in mats0)
    kv_bytes = L * layer_bytes(POS)
    step_bytes = kv_bytes + w_bytes
    peaks = load_peaks()
    layer_ms = ms / L
    achieved = step_bytes / L / (layer_ms * 1e-3) / 1e9
    return {
        "metric": "attention block (Q8_K + Wq/Wk/Wv + attention + Wo) GB/s of KV + weights @7B ctx 32k",
        "value": round(step_bytes / (ms * 1e-3) / 1e9, 1), "unit": "GB/s", "ms_per_step": round(ms, 5),
        "steps": steps, "layers": L, "weight_bytes_per_step": int(w_bytes), "kv_bytes_per_step": int(kv_bytes),
        "weights": "Q4_K wq/wk/wo, Q6_K wv (seeded synthetic GGUF blocks)",
        "e2e": {"value": round(step_bytes / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s", "ms_per_step": round(e2e_ms, 4),
                "h2d_bytes_per_step": L * E * 4, "d2h_bytes_per_step": L * E * 4},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"],
                     "peak_source": peaks["source"], "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                     "kernels": "qmatvec_kernel (QKV) + attn_decode_kernel + split_merge_kernel + qmatvec_kernel (Wo)"},
        "gpu_launches": steps * L * 4,
        "clocks": clk,
        "_cpu_proj_ms": cpu_proj_ms,
    }


# config 5: Qwen2.5-3B-shaped batched decode of many independent sequences
B_SEQS, B_LAYERS, B_H, B_G = 64, 36, 16, 2
B_KVD = B_G * D


def batched_lengths() -> np.ndarray:
    """Cached positions of the 64 sequences, ~U{1024..32768}, seeded."""
    return np.random.default_rng(5).integers(1024, 32769, B_SEQS)


def batched_seq_bytes(length: int) -> int:
    """Algorithmic bytes of one sequence's decode step over all layers."""
    return B_LAYERS * (2 * (length + 1) * B_KVD * 4 + 2 * B_H * D * 4 + 2 * B_KVD * 4)


def run_batched(args, rank: int, world: int, dist, peaks) -> dict | None:
    """Config 5: 64 sequences of ragged length decode one token each through 36
    layers (3B shape). The sequences are split over the GPUs longest-first
    (kore_b200.shard.assign_sequences); each GPU holds only its sequences'
    pages and runs one batched decode launch per layer, with no data-path
    collective. value = all ranks' algorithmic bytes / max-over-ranks time."""
    import torch
    import kore_b200 as K
    from kore_b200.shard import assign_sequences
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    lengths = batched_lengths()
    mine = assign_sequences(lengths, world)[rank]
    P = 256
    n_pages = sum((int(lengths[i]) + 1 + P - 1) // P for i in mine)
    ctx = K.KoreCuda(B_LAYERS, B_H, B_G, D, int(lengths.max()) + 1, max_seqs=len(mine), n_pages=n_pages,
                     device=dev.index)
    stream = torch.cuda.Stream(device=dev)
    ctx.set_stream(stream.cuda_stream)
    gen = torch.Generator(device=dev)
    n = len(mine)
    pos = np.array([int(lengths[i]) for i in mine], np.int32)
    seqs = np.arange(n, dtype=np.int32)
    with torch.cuda.stream(stream):
        # one seeded block of rows per layer; every sequence appends its own
        # prefix of it into its own pages
        for layer in range(B_LAYERS):
            gen.manual_seed(100000 + layer)
            k = torch.randn(int(lengths.max()), B_KVD, device=dev, generator=gen)
            v = torch.randn(int(lengths.max()), B_KVD, device=dev, generator=gen)
            for j in range(len(mine)):
                ctx.append_dev(j, layer, 0, int(pos[j]), k[:int(pos[j])], v[:int(pos[j])])
            del k, v
        gen.manual_seed(11 + rank)
        q = torch.randn(B_LAYERS, n, B_H * D, device=dev, generator=gen)
        kn = torch.randn(B_LAYERS, n, B_KVD, device=dev, generator=gen)
        vn = torch.randn(B_LAYERS, n, B_KVD, device=dev, generator=gen)
        out = torch.empty(B_LAYERS, n, B_H * D, device=dev)
    ctx.sync()

    def step():
        for layer in range(B_LAYERS):
            ctx.decode_batch_dev(layer, seqs, pos, q[layer], kn[layer], vn[layer], out[layer])

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(dev)

    with torch.cuda.stream(stream):
        for _ in range(3):
            step()
    ctx.sync()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    with torch.cuda.stream(stream):
        graph.replay()
    ctx.sync()
    steps = args.batched_steps
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(steps):
            graph.replay()
        e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / steps
    barrier()
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = t.item()
    del graph
    ctx.close()
    if rank != 0:
        return None
    total = sum(batched_seq_bytes(int(x)) for x in lengths)
    gbs = total / (ms * 1e-3) / 1e9
    return {
        "metric": "batched decode attn HBM GB/s (cfg5: 3B shape, 64 sequences, 36 layers)",
        "value": round(gbs, 1), "unit": "GB/s", "n_gpus": world, "steps": steps, "warmup": 3,
        "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong" if world > 1 else "weak",
        "config": {"workload": "cfg5: 64 sequences, cached lengths ~U{1024..32768} (seed 5), 16Q/2KV heads, "
                               "d128, 36 layers, 256-token pages, one token per sequence per step",
                   "kv_bytes_per_step": int(total), "assignment": "longest-first to the least-loaded GPU",
                   "cache": "per layer one seeded N(0,1) block; each sequence holds its prefix in its own pages",
                   "l2": f"{total / 1e9:.0f} GB of KV per step > L2, no flush needed"},
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": round(peaks["hbm_gbs"] * world, 1),
                     "peak_source": peaks["source"], "unit": "GB/s",
                     "frac": round(gbs / (peaks["hbm_gbs"] * world), 4),
                     "note": "peak = measured HBM GB/s x GPUs"},
        "gpu_launches": steps * B_LAYERS * 2,
    }


def prefill_pairs(pos0: int, n: int) -> int:
    """Unmasked (query, key) pairs of a causal chunk: sum over z of pos0 + z + 1."""
    return n * (pos0 + 1) + n * (n - 1) // 2


def run_prefill(args, dev, peaks) -> dict:
    """Config 3: a 2048-token chunk appended onto 4096 cached rows, 28 layers,
    7B shape; one step = the chunk through every layer (append, operand
    split, tensor-core attention), re-run at the same positions each step."""
    import torch
    import kore_b200 as K
    P0, N, LP = 4096, 2048, args.prefill_layers
    ctx = K.KoreCuda(LP, H, G, D, P0 + N, device=dev.index)
    stream = torch.cuda.Stream(device=dev)
    ctx.set_stream(stream.cuda_stream)
    gen = torch.Generator(device=dev)
    with torch.cuda.stream(stream):
        for layer in range(LP):
            gen.manual_seed(2000 + layer)
            k = torch.randn(P0, KVD, device=dev, generator=gen)
            v = torch.randn(P0, KVD, device=dev, generator=gen)
            ctx.append_dev(0, layer, 0, P0, k, v)
        gen.manual_seed(9)
        q = torch.randn(LP, N, H * D, device=dev, generator=gen)
        kc = torch.randn(LP, N, KVD, device=dev, generator=gen)
        vc = torch.randn(LP, N, KVD, device=dev, generator=gen)
        out = torch.empty(LP, N, H * D, device=dev)
    ctx.sync()

    def step():
        for layer in range(LP):
            ctx.prefill_dev(0, layer, P0, N, q[layer], kc[layer], vc[layer], out[layer])

    with torch.cuda.stream(stream):
        for _ in range(2):
            step()
    ctx.sync()
    steps = args.prefill_steps
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(steps):
            step()
        e1.record(stream)
    e1.synchronize()
    ctx.sync()
    ms = e0.elapsed_time(e1) / steps
    flops = 4 * D * prefill_pairs(P0, N) * H * LP
    tflops = flops / (ms * 1e-3) / 1e12
    ctx.close()
    # the tensor pipe runs three bf16 MMAs per fp32-accurate product
    peak_eq = peaks["bf16_tflops"] / 3
    return {"metric": "prefill attn TFLOP/s (7B, 2048-token chunk onto 4096, 28 layers)",
            "value": round(tflops, 1), "unit": "TFLOP/s", "ms_per_step": round(ms, 4), "steps": steps,
            "layers": LP, "flop_per_step": flops,
            "roofline": {"bound": "tensor", "achieved": round(tflops, 1), "peak": round(peak_eq, 1),
                         "unit": "TFLOP/s", "frac": round(tflops / peak_eq, 4), "peak_source": peaks["source"],
                         "peak_note": "measured bf16 dense peak / 3: each fp32-accurate product is three bf16 "
                                      "MMAs (hi*hi + hi*mid + mid*hi)"},
            "kernels": "kv_append_kernel + kv_split_kernel + prefill_kernel (tcgen05, TMEM)"}


def load_peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            j = json.load(f)
        return {"hbm_gbs": float(j["hbm_gbs"]), "bf16_tflops": float(j["bf16_tflops"]), "source": "measured"}
    except (OSError, KeyError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def load_traffic():
    """DRAM bytes per decode launch from the committed ncu summary, if any."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(p) as f:
            return json.load(f).get("attn_decode_cfg4_bytes_per_launch")
    except (OSError, ValueError):
        return None


# ---------------------------------------------------------------- reference arm (CPU)

def _ref_layer_engines(n: int, threads: int = 1):
    from oracle import oracle as O
    engines = []
    for i in range(n):
        e = O.RefLayer(H, G, D, CTX, threads=threads)
        g = np.random.default_rng(100 + i)
        for p0 in range(0, POS, 4096):
            k = g.standard_normal((4096, KVD), dtype=np.float32)
            v = g.standard_normal((4096, KVD), dtype=np.float32)
            e.fill(p0, k, v)
        engines.append(e)
    return engines


def _ref_decode_ms(e, pos: int, reps: int = 1) -> float:
    from oracle import oracle as O
    q, k, v = O.seeded_inputs(5, (H * D,), (KVD,), (KVD,))
    t0 = time.perf_counter()
    for _ in range(reps):
        e.decode(pos, q, k, v)
    return (time.perf_counter() - t0) * 1e3 / reps


def cpu_baseline_sample() -> dict:
    """kore's own decode attention (forward() of the compiled reference) on 1
    core, one layer at position 32768, minus the same forward() at position 0
    (embedding, norms and zero-weight projections, i.e. everything that is
    not attention)."""
    from oracle import oracle as O
    if not O.ref_available():
        return {"value": None, "unavailable": "oracle/_ref not built"}
    e = _ref_layer_engines(1)[0]
    base = _ref_decode_ms(e, 0, reps=3)
    t = min(_ref_decode_ms(e, POS) for _ in range(3))
    att = max(t - base, 1e-6)
    return {"value": round(layer_bytes(POS) / (att * 1e-3) / 1e9, 3), "unit": "GB/s", "cores": 1,
            "kind": "reference", "attention_ms": round(att, 3),
            "sample": f"1 of 28 layers, decode at pos {POS}, kore forward() best of 3 = {t:.1f} ms "
                      f"minus forward() at pos 0 = {base:.1f} ms; attention {att:.1f} ms"}


def run_reference(args, rank: int, world: int) -> dict | None:
    if rank != 0:
        return None
    from oracle import oracle as O
    if not O.ref_available():
        return {"impl": "reference", "unavailable": "oracle/_ref/libkore_ref.so not built (needs the reference sources)"}
    cores = len(os.sched_getaffinity(0))
    T = max(1, min(cores, L))
    engines = _ref_layer_engines(T)
    base = _ref_decode_ms(engines[0], 0, reps=3)
    from oracle import oracle as O2
    q, k, v = O2.seeded_inputs(5, (H * D,), (KVD,), (KVD,))

    def one_step():
        # T layers at once, one per core: kore's attention is single-threaded
        ths = [threading.Thread(target=e.decode, args=(POS, q, k, v)) for e in engines]
        t0 = time.perf_counter()
        for th in ths:
            th.start()
        for th in ths:
            th.join()
        return (time.perf_counter() - t0) * 1e3

    budget_s = 150.0
    first = one_step()
    n_total = args.warmup + args.steps
    steps = max(1, min(args.steps, int(budget_s * 1e3 / max(first, 1.0)) - min(args.warmup, 2)))
    warm = min(args.warmup, 2)
    for _ in range(max(0, warm - 1)):
        one_step()
    times = [one_step() for _ in range(steps)]
    ms = sum(times) / len(times)
    att_ms = max(ms - base, 1e-6)   # non-attention part of forward() runs in parallel too
    v_gbs = T * layer_bytes(POS) / (att_ms * 1e-3) / 1e9
    return {
        "impl": "reference", "metric": "decode attn HBM GB/s @7B ctx 32k (28 layers, 28Q/4KV, d128, fp32 KV)",
        "value": round(v_gbs, 3), "unit": "GB/s", "n_gpus": world, "steps": steps, "warmup": warm,
        "steps_requested": args.steps, "ms_per_step": round(att_ms, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1))",
        "config": {"workload": "cfg4: Qwen2.5-7B-shaped decode at position 32768, 28 layers, batch 1"},
        "cpu_baseline": {"value": round(v_gbs, 3), "unit": "GB/s", "cores": T, "kind": "reference",
                         "sample": f"each step: {T} of the 28 layers decoded concurrently, one kore forward() "
                                   f"per core (kore's attention is single-threaded), minus forward() at pos 0 "
                                   f"({base:.1f} ms); {steps} of {n_total} requested steps within {budget_s:.0f} s"},
        "e2e": {"value": round(v_gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# ---------------------------------------------------------------- main

def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    dist = None
    if args.impl == "reference":
        line = run_reference(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0))))
    if args.prefill_only:
        import torch
        print(json.dumps(run_prefill(args, torch.device("cuda", 0), load_peaks())), flush=True)
        return
    if args.block_only:
        print(json.dumps(run_block_only(args)), flush=True)
        return
    try:
        line = run_ours(args, rank, world, dist)
        if not args.no_batched:
            import torch
            batched = run_batched(args, rank, world, dist, load_peaks())
            if line is not None:
                line["batched"] = batched
        if line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
