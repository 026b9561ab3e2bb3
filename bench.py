"""bench.py — decode attention throughput of the B200 kore path.

Headline workload (the metric's "@7B ctx 32k"):
Qwen2.5-7B-shaped attention, 28 layers, 28 query / 4 KV heads, head_dim 128,
one sequence, fp32 KV cache of 32768 seeded N(0,1) rows per layer (3.5 GiB,
far larger than the 126 MB L2, so no L2 flush is needed between steps). One
step = one decode token through all 28 layers: RoPE of q/k at position 32768,
append of k/v, attention over positions 0..32768.

  value  device-resident: q/k/v already in HBM, CUDA events on the context's
         stream around K replays of a CUDA graph holding one step; max over
         ranks; GB/s of algorithmic bytes
         (per layer: 2*(pos+1)*512*4 K/V + 2*28*128*4 q/out + 2*512*4 append).
  e2e    the same steps through the host-buffer C entry point
         kore_cuda_attn_decode (kore's call: host q/k/v in, host out back;
         kore_cuda_attn_decode_sharded at N > 1), wall clock, copies included.
  parity at N = 1 layer 0's output against kore's own forward() (the
         reference compiled in place) on the same cache and inputs, inside the
         CPU-baseline leg; at N > 1 against the unsharded decode of the same
         layer rebuilt on each rank's GPU. A failed check exits non-zero.
At N > 1 the KV positions are split over the GPUs by page (round robin); each
layer's partial outputs and log-sum-exps are pushed to every peer over NVLink
peer memory and merged on every rank (kore_cuda_attn_decode_sharded_dev), one
exchange per layer. The cache is fixed (strong scaling).

Further lines on the same JSON object (N = 1 unless stated): ``cfg1`` (the
0.5B layer: prefill 128, then 64 decodes; microseconds per call), ``cfg2``
(7B, 28 layers, decode at 8192), ``attn_block`` (the attention block with its
quantised projections), ``prefill`` (config 3, tensor cores),
``decode_step`` (kore's whole decode step on the device: 7B-shaped synthetic
weights, the headline's cache; tokens/s), ``prefill_model`` (kore's
forward_batch for a 2048-token prompt through the same model on the device;
tokens/s) and ``batched`` (config 5, every N).

``--impl reference`` times kore's own CPU attention (the reference compiled
in place, oracle/_ref) on this host: full 28-layer steps of kore.cpp forward()
per layer on its fp32 cache, the layers fanned over the host's cores.
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
ABS_TOL, REL_TOL = 2e-3, 1e-3   # per head: max-abs, and max-abs / max |reference|


def layer_bytes(pos: int, h: int = H, kvd: int = KVD, d: int = D) -> int:
    return 2 * (pos + 1) * kvd * 4 + 2 * h * d * 4 + 2 * kvd * 4


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
    ap.add_argument("--no-cfg12", action="store_true", help="skip the config-1 and config-2 lines")
    ap.add_argument("--no-step", action="store_true", help="skip the whole-decode-step line")
    ap.add_argument("--step-only", action="store_true", help="measure only the whole decode step (development)")
    ap.add_argument("--prefill-model-only", action="store_true", help="measure only the whole-model prefill")
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


def head_errors(out, ref):
    """Worst (max-abs, max-abs / max |ref|) over the heads (rows of D values)."""
    o = np.asarray(out, np.float64).reshape(-1, D)
    r = np.asarray(ref, np.float64).reshape(-1, D)
    err = np.abs(o - r).max(axis=1)
    mag = np.maximum(np.abs(r).max(axis=1), 1e-30)
    return float(err.max()), float((err / mag).max())


def parity_entry(out, ref, against: str) -> dict:
    a, r = head_errors(out, ref)
    ok = bool(np.isfinite(np.asarray(out)).all()) and a <= ABS_TOL and r <= REL_TOL
    return {"max_abs": a, "max_rel": r, "ok": ok, "tol": {"abs": ABS_TOL, "rel": REL_TOL}, "against": against}


def cfg4_config(world: int, pos: int = None, layers: int = None) -> dict:
    pos = POS if pos is None else pos
    layers = L if layers is None else layers
    name = "cfg4" if pos == 32768 else ("cfg2" if pos == 8192 else "decode")
    return {"workload": f"{name}: Qwen2.5-7B-shaped decode at position {pos}, {layers} layers, batch 1",
            "kv_bytes_per_step": layers * layer_bytes(pos), "l2": f"inputs {layers * layer_bytes(pos) / 2**30:.2f} GiB "
            "> L2, no flush needed",
            "kv_split": f"pages round-robin over {world} GPU(s)" if world > 1 else "none"}


def layer_rows(torch, dev, layer: int, n: int):
    """The seeded N(0,1) pre-RoPE k and v rows of one layer, generated on `dev`."""
    gen = torch.Generator(device=dev)
    gen.manual_seed(1000 + layer)
    k = torch.randn(n, KVD, device=dev, generator=gen)
    v = torch.randn(n, KVD, device=dev, generator=gen)
    return k, v


# ---------------------------------------------------------------- our arm: 7B decode (cfg4, cfg2)

def run_decode(args, rank: int, world: int, dist, pos: int, layers: int, steps: int, e2e_steps: int,
               want_block: bool) -> dict | None:
    """Decode at `pos` through `layers` layers of the 7B shape, at N = world
    GPUs (the KV positions split by page). Returns rank 0's line."""
    import torch
    import kore_b200 as K

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    ctx = K.KoreCuda(layers, H, G, D, pos + 1, device=dev.index, shard_rank=rank, shard_count=world)
    # the context runs on a torch-owned stream, so tensors used on it (and by
    # NCCL) outlive nothing they depend on when the context is closed
    stream = torch.cuda.Stream(device=dev)
    ctx.set_stream(stream.cuda_stream)

    # seeded N(0,1) cache: all rows generated on the device per layer; each
    # shard stores the rows of the pages it holds
    gen = torch.Generator(device=dev)
    with torch.cuda.stream(stream):
        for layer in range(layers):
            k, v = layer_rows(torch, dev, layer, pos)
            ctx.append_dev(0, layer, 0, pos, k, v)
            del k, v
        gen.manual_seed(7)
        q = torch.randn(layers, H * D, device=dev, generator=gen)
        kn = torch.randn(layers, KVD, device=dev, generator=gen)
        vn = torch.randn(layers, KVD, device=dev, generator=gen)
        out = torch.empty(layers, H * D, device=dev)
        part = torch.empty(layers, ctx.part_floats, device=dev)
    ctx.sync()

    if world > 1:
        from kore_b200.shard import exchange_handles
        exchange_handles(ctx, dist)     # exchange buffers mapped over CUDA IPC

    def step():
        for layer in range(layers):
            if world == 1:
                ctx.decode_dev(0, layer, pos, q[layer], kn[layer], vn[layer], out[layer])
            else:
                # partial on this rank's pages, pushed to the peers over NVLink, merged on every rank
                ctx.decode_sharded_dev(0, layer, pos, q[layer], kn[layer], vn[layer], out[layer])

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
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

    clocks = ClockSampler(dev.index)
    clocks.start()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    barrier()
    t_begin = time.time()
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(steps):
            graph.replay()
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
    n_ev = min(steps, 50)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n_ev * layers)]
    with torch.cuda.stream(stream):
        for s in range(n_ev):
            for layer in range(layers):
                a, b = evs[s * layers + layer]
                a.record(stream)
                if world == 1:
                    ctx.decode_dev(0, layer, pos, q[layer], kn[layer], vn[layer], out[layer])
                else:
                    ctx.decode_partial_dev(0, layer, pos, q[layer], kn[layer], vn[layer], part[layer])
                b.record(stream)
    torch.cuda.synchronize(dev)
    iso_ms = sum(a.elapsed_time(b) for a, b in evs) / len(evs)

    # end to end through the host-buffer entry point (kore's own call shape):
    # q/k/v in from host memory, the merged output back into host memory, one
    # C-ABI call per layer with kore's raw pointers (the library copies in and
    # out inside each call); the numpy wrapper's cost is reported beside it
    hq, hk, hv = q.cpu().numpy(), kn.cpu().numpy(), vn.cpu().numpy()
    ho = np.empty((layers, H * D), np.float32)
    c_dec = ctx.c_call("kore_cuda_attn_decode" if world == 1 else "kore_cuda_attn_decode_sharded")
    ptrs = [(hq[l].ctypes.data, hk[l].ctypes.data, hv[l].ctypes.data, ho[l].ctypes.data) for l in range(layers)]

    def host_step():
        for layer in range(layers):
            qa, ka, va, oa = ptrs[layer]
            c_dec(0, layer, pos, qa, ka, va, oa)
    host_step()
    barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        host_step()
    e2e_ms = (time.perf_counter() - t0) * 1e3 / e2e_steps
    barrier()
    wrap = ctx.decode if world == 1 else ctx.decode_sharded
    n_w = max(3, e2e_steps // 10)
    t0 = time.perf_counter()
    for _ in range(n_w):
        for layer in range(layers):
            ho[layer] = wrap(0, layer, pos, hq[layer], hk[layer], hv[layer]).reshape(-1)
    wrapped_us = (time.perf_counter() - t0) * 1e6 / (n_w * layers)
    barrier()

    # where a host-buffer call's time goes (one GPU): the same layer calls with
    # the inputs already on the device and a synchronisation after each (no
    # staging), and the synchronisation alone (the error word's copy back and
    # the stream wait), each per layer
    breakdown = None
    if world == 1:
        n_b = max(5, e2e_steps // 4)
        with torch.cuda.stream(stream):
            t0 = time.perf_counter()
            for _ in range(n_b):
                for layer in range(layers):
                    ctx.decode_dev(0, layer, pos, q[layer], kn[layer], vn[layer], out[layer])
                    ctx.sync()
            dev_sync_us = (time.perf_counter() - t0) * 1e6 / (n_b * layers)
            t0 = time.perf_counter()
            for _ in range(n_b * layers):
                ctx.sync()
            sync_us = (time.perf_counter() - t0) * 1e6 / (n_b * layers)
        breakdown = {"host_call_us": round(e2e_ms * 1e3 / layers, 2),
                     "python_wrapper_call_us": round(wrapped_us, 2),
                     "device_inputs_call_plus_sync_us": round(dev_sync_us, 2),
                     "sync_alone_us": round(sync_us, 2),
                     "staging_us": round(e2e_ms * 1e3 / layers - dev_sync_us, 2),
                     "note": "per layer: host_call = kore_cuda_attn_decode with host q/k/v/out (raw pointers, as "
                             "kore calls it); python_wrapper_call = the same through KoreCuda.decode (numpy "
                             "conversions and a new output array per call); the next figure is "
                             "kore_cuda_attn_decode_dev (inputs in HBM) + kore_cuda_sync after each call; sync_alone "
                             "is kore_cuda_sync with nothing queued (error-word copy + stream wait); staging = "
                             "host_call - the second figure (host copies, the input kernel, the output copy)"}

    # parity at N > 1: layer 0 rebuilt unsharded on this GPU from the same
    # seeds, decoded with the same q/k/v, against the merged sharded output
    parity = None
    if world > 1:
        full = K.KoreCuda(1, H, G, D, pos + 1, device=dev.index)
        k0, v0 = layer_rows(torch, dev, 0, pos)
        full.append_dev(0, 0, 0, pos, k0, v0)
        del k0, v0
        ref = torch.empty(H * D, device=dev)
        full.decode_dev(0, 0, pos, q[0], kn[0], vn[0], ref)
        full.sync()
        full.close()
        parity = parity_entry(ho[0], ref.cpu().numpy(), "the unsharded decode of layer 0 on the same GPU "
                              "(same seeded cache and q/k/v), on every rank")

    t = torch.tensor([ms, iso_ms, e2e_ms, 0.0 if parity is None or parity["ok"] else 1.0,
                      0.0 if parity is None else parity["max_abs"], 0.0 if parity is None else parity["max_rel"]],
                     device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, iso_ms, e2e_ms, bad, pa, pr = t.tolist()
    if parity is not None:
        parity.update(max_abs=pa, max_rel=pr, ok=bad == 0.0, ranks=world)

    block = None
    if want_block and world == 1 and not args.no_block:
        block = run_block(args, ctx, stream, dev)
    layer0 = ho[0].copy()
    ctx.close()
    if rank != 0:
        return None

    step_bytes = layers * layer_bytes(pos)
    ms_step = ms / steps
    gbs = step_bytes / (ms_step * 1e-3) / 1e9
    e2e_gbs = step_bytes / (e2e_ms * 1e-3) / 1e9
    peaks = load_peaks()
    launch_bytes = layer_bytes(pos) / world
    layer_ms = ms_step / layers          # one layer's decode (+ split merge or exchange) inside the timed region
    achieved = launch_bytes / (layer_ms * 1e-3) / 1e9
    line = {
        "metric": f"decode attn HBM GB/s @7B ctx {pos // 1024}k ({layers} layers, 28Q/4KV, d128, fp32 KV)",
        "value": round(gbs, 1), "unit": "GB/s", "n_gpus": world, "steps": steps, "warmup": max(3, args.warmup),
        "ms_per_step": round(ms_step, 5), "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1) q/k/v and KV cache)",
        "config": cfg4_config(world, pos, layers),
        "e2e": {"value": round(e2e_gbs, 1), "unit": "GB/s", "ms_per_step": round(e2e_ms, 4),
                "h2d_bytes_per_step": layers * (H * D + 2 * KVD) * 4, "d2h_bytes_per_step": layers * H * D * 4,
                "call": "kore_cuda_attn_decode" if world == 1 else "kore_cuda_attn_decode_sharded",
                "breakdown": breakdown},
        "roofline": {"bound": "hbm",
                     "kernel": "attn_decode_kernel<128,7,8,8,3> with " + (
                         "its split merge in the same launch" if world == 1
                         else "its split merge and the peer exchange in the same launch"),
                     "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "peak_source": peaks["source"],
                     "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                     "traffic": load_traffic() if pos == 32768 and world == 1 else None,
                     "launch_ms": round(layer_ms, 5), "launch_ms_isolated": round(iso_ms, 5),
                     "algorithmic_bytes_per_launch": int(launch_bytes),
                     "timing": "launch_ms = timed region / (steps x layers), CUDA events on the context stream; "
                               "launch_ms_isolated = events around each layer's call (no inter-layer overlap)"},
        "gpu_launches": steps * layers * (1 + merge_launch(world)),
        "clocks": clk,
    }
    if world == 1:
        if not args.no_cpu_baseline:
            cb, par = cpu_baseline_sample(pos, layer0, hq[0], hk[0], hv[0])
            line["cpu_baseline"] = cb
            if par is not None:
                parity = par
    if parity is not None:
        line["parity"] = parity
    if block is not None:
        proj_ms = block.pop("_cpu_proj_ms", None)
        att = line.get("cpu_baseline", {}).get("attention_ms")
        if proj_ms is not None and att is not None:
            per_layer = block["weight_bytes_per_step"] / layers + layer_bytes(pos)
            block["cpu_baseline"] = {
                "value": round(per_layer / ((att + proj_ms) * 1e-3) / 1e9, 3), "unit": "GB/s", "cores": 1,
                "kind": "reference",
                "sample": f"1 of 28 layers: kore's attention at pos {pos} ({att:.1f} ms, as cpu_baseline) + "
                          f"kore's quantize_row_q8_K + matvec_mt of Wq, Wk, Wv, Wo on 1 thread "
                          f"(best of 3, {proj_ms:.2f} ms)"}
        line["attn_block"] = block
    return line


def run_block_only(args) -> dict:
    """The attention-block line alone, on a context set up as run_decode sets it up."""
    import torch
    import kore_b200 as K

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    ctx = K.KoreCuda(L, H, G, D, CTX, device=0)
    stream = torch.cuda.Stream(device=dev)
    ctx.set_stream(stream.cuda_stream)
    with torch.cuda.stream(stream):
        for layer in range(L):
            k, v = layer_rows(torch, dev, layer, POS)
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

    warm = max(3, args.warmup)
    with torch.cuda.stream(stream):
        for _ in range(warm):
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
    # (raw host pointers, as kore passes them)
    hx = xb.cpu().numpy()
    hob = np.empty_like(hx)
    c_blk = ctx.c_call("kore_cuda_attn_block_decode")
    bptr = [(hx[l].ctypes.data, hob[l].ctypes.data) for l in range(L)]
    for layer in range(L):
        c_blk(0, layer, POS, *bptr[layer])
    n_e2e = max(1, args.e2e_steps // 4)
    t0 = time.perf_counter()
    for _ in range(n_e2e):
        for layer in range(L):
            c_blk(0, layer, POS, *bptr[layer])
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
        "steps": steps, "warmup": warm, "layers": L, "weight_bytes_per_step": int(w_bytes),
        "kv_bytes_per_step": int(kv_bytes), "weights": "Q4_K wq/wk/wo, Q6_K wv (seeded synthetic GGUF blocks)",
        "e2e": {"value": round(step_bytes / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s", "ms_per_step": round(e2e_ms, 4),
                "h2d_bytes_per_step": L * E * 4, "d2h_bytes_per_step": L * E * 4},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"],
                     "peak_source": peaks["source"], "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                     "kernels": "qmatvec_kernel (QKV) + attn_decode_kernel (split merge in the launch) + qmatvec_kernel (Wo)"},
        "gpu_launches": steps * L * (3 + merge_launch()),
        "clocks": clk,
        "_cpu_proj_ms": cpu_proj_ms,
    }


# ---------------------------------------------------------------- config 1: the 0.5B layer

C1_H, C1_G, C1_D, C1_PRE, C1_DEC = 14, 2, 64, 128, 64


def run_cfg1(args) -> dict:
    """Config 1: one Qwen2.5-0.5B-shaped attention layer (14Q/2KV, d 64):
    prefill 128 tokens at positions 0..127, then 64 decode steps at 128..191,
    fresh seeded N(0,1) q/k/v per call. One step = that whole workload (65
    calls), re-run at the same positions (the prefill from position 0
    overwrites the cache, as kore's re-prefill does). Latency-bound: the
    line reports microseconds per call. `value`: device-resident inputs, one
    CUDA graph replay per step, CUDA events; `e2e`: kore's host-buffer calls
    (kore_cuda_attn_prefill / kore_cuda_attn_decode), each returning once its
    output is on the host, wall clock."""
    import torch
    import kore_b200 as K

    dev = torch.device("cuda", 0)
    hd, kvd = C1_H * C1_D, C1_G * C1_D
    n_calls = 1 + C1_DEC
    ctx = K.KoreCuda(1, C1_H, C1_G, C1_D, C1_PRE + C1_DEC, device=0)
    stream = torch.cuda.Stream(device=dev)
    ctx.set_stream(stream.cuda_stream)
    rng = np.random.default_rng(12345)
    hq = rng.standard_normal((C1_PRE + C1_DEC, hd), dtype=np.float32)
    hk = rng.standard_normal((C1_PRE + C1_DEC, kvd), dtype=np.float32)
    hv = rng.standard_normal((C1_PRE + C1_DEC, kvd), dtype=np.float32)
    with torch.cuda.stream(stream):
        q, k, v = (torch.from_numpy(a).to(dev) for a in (hq, hk, hv))
        out = torch.empty(C1_PRE + C1_DEC, hd, device=dev)

    def step():
        ctx.prefill_dev(0, 0, 0, C1_PRE, q[:C1_PRE], k[:C1_PRE], v[:C1_PRE], out[:C1_PRE])
        for i in range(C1_DEC):
            p = C1_PRE + i
            ctx.decode_dev(0, 0, p, q[p], k[p], v[p], out[p])

    warm = max(3, args.warmup)
    with torch.cuda.stream(stream):
        for _ in range(warm):
            step()
    ctx.sync()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    with torch.cuda.stream(stream):
        graph.replay()
    ctx.sync()
    steps = max(20, args.steps // 10)
    clocks = ClockSampler(0)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    t_begin = time.time()
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(steps):
            graph.replay()
        e1.record(stream)
    e1.synchronize()
    t_end = time.time()
    clk = clocks.stop(t_begin, t_end)
    ms = e0.elapsed_time(e1) / steps
    del graph
    # the pieces, device side: the prefill call alone and one decode call
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(n_calls + 1)]
    with torch.cuda.stream(stream):
        ev[0].record(stream)
        ctx.prefill_dev(0, 0, 0, C1_PRE, q[:C1_PRE], k[:C1_PRE], v[:C1_PRE], out[:C1_PRE])
        ev[1].record(stream)
        for i in range(C1_DEC):
            p = C1_PRE + i
            ctx.decode_dev(0, 0, p, q[p], k[p], v[p], out[p])
            ev[2 + i].record(stream)
    torch.cuda.synchronize(dev)
    pre_us = ev[0].elapsed_time(ev[1]) * 1e3
    dec_us = ev[1].elapsed_time(ev[-1]) * 1e3 / C1_DEC
    # end to end: kore's host-buffer calls, with raw host pointers as kore
    # passes them (outputs into one host array)
    ho = np.empty((C1_PRE + C1_DEC, hd), np.float32)
    c_pre, c_dec = ctx.c_call("kore_cuda_attn_prefill"), ctx.c_call("kore_cuda_attn_decode")
    row = lambda a, i: a.ctypes.data + i * a.strides[0]  # noqa: E731

    def e2e_once():
        c_pre(0, 0, 0, C1_PRE, row(hq, 0), row(hk, 0), row(hv, 0), row(ho, 0))
        for i in range(C1_DEC):
            p = C1_PRE + i
            c_dec(0, 0, p, row(hq, p), row(hk, p), row(hv, p), row(ho, p))
    for _ in range(3):
        e2e_once()
    n_e2e = 20
    t0 = time.perf_counter()
    for _ in range(n_e2e):
        e2e_once()
    e2e_ms = (time.perf_counter() - t0) * 1e3 / n_e2e
    ctx.close()
    line = {
        "metric": "cfg1 attention latency, microseconds per call (0.5B layer: prefill 128, then 64 decodes)",
        "value": round(ms * 1e3 / n_calls, 2), "unit": "us/call", "higher_is_better": False,
        "steps": steps, "warmup": warm, "ms_per_step": round(ms, 5), "dtype": "f32",
        "data": "synthetic (seeded N(0,1) q/k/v, numpy seed 12345)",
        "config": {"workload": "cfg1: Qwen2.5-0.5B-shaped attention layer, 14Q/2KV, d64, prefill 128 tokens at "
                               "0..127 then 64 decode steps at 128..191, RoPE theta 1e6", "calls_per_step": n_calls},
        "device_us": {"prefill_128": round(pre_us, 2), "decode_mean": round(dec_us, 2),
                      "timing": "device: CUDA graph of one step (65 calls), events around K replays; the pieces "
                                "from events around each call of one ungraphed step"},
        "e2e": {"value": round(e2e_ms * 1e3 / n_calls, 2), "unit": "us/call", "ms_per_step": round(e2e_ms, 4),
                "h2d_bytes_per_step": (C1_PRE + C1_DEC) * (hd + 2 * kvd) * 4,
                "d2h_bytes_per_step": (C1_PRE + C1_DEC) * hd * 4},
        "roofline": {"bound": "latency", "note": "29.6 MFLOP of prefill and <= 0.2 MB per decode: launch and "
                                                 "dependency latency bound, far from HBM or tensor limits"},
        # prefill: append, operand split, tensor-core kernel; each decode: the
        # decode kernel with its split merge (positions 128..191 take 4-6 splits)
        "gpu_launches": steps * (3 + C1_DEC * (1 + merge_launch())),
        "clocks": clk,
    }
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = cfg1_cpu_baseline(hq, hk, hv)
    return line


def cfg1_cpu_baseline(hq, hk, hv) -> dict:
    """kore's own attention (forward_batch() per prompt token, then forward()
    per decode token; the reference compiled in place) on one core for the
    same 65 calls, minus the non-attention part of forward() (its time at
    position 0), microseconds per call."""
    from oracle import oracle as O
    if not O.ref_available():
        return {"value": None, "unavailable": "oracle/_ref not built"}
    e = O.RefLayer(C1_H, C1_G, C1_D, C1_PRE + C1_DEC)
    best = None
    for _ in range(3):
        t0 = time.perf_counter()
        e.prefill(0, hq[:C1_PRE], hk[:C1_PRE], hv[:C1_PRE])
        for i in range(C1_DEC):
            p = C1_PRE + i
            e.decode(p, hq[p], hk[p], hv[p])
        t = (time.perf_counter() - t0) * 1e3
        best = t if best is None else min(best, t)
    # the non-attention part of each kind of call (its time at position 0,
    # one key): forward_batch() for the prompt tokens, forward() for the decodes
    t0 = time.perf_counter()
    for _ in range(20):
        e.prefill(0, hq[:1], hk[:1], hv[:1])
    base_pre = (time.perf_counter() - t0) * 1e3 / 20
    t0 = time.perf_counter()
    for _ in range(20):
        e.decode(0, hq[0], hk[0], hv[0])
    base_dec = (time.perf_counter() - t0) * 1e3 / 20
    att = max(best - C1_PRE * base_pre - C1_DEC * base_dec, 1e-6)
    return {"value": round(att * 1e3 / (1 + C1_DEC), 2), "unit": "us/call", "cores": 1, "kind": "reference",
            "ms_per_step": round(att, 3),
            "sample": f"the whole workload, best of 3: {best:.2f} ms, minus the non-attention part of each call "
                      f"(its time at position 0: {C1_PRE} x {base_pre:.3f} ms of forward_batch, {C1_DEC} x "
                      f"{base_dec:.3f} ms of forward); kore's prefill token by token (forward_batch nb = 1, the same "
                      f"attention arithmetic per token); per call = attention time / 65 calls"}


# ---------------------------------------------------------------- the whole decode step (device-resident)

S_FF, S_VOCAB = 18944, 152064   # Qwen2.5-7B feed-forward width and vocabulary


def step_model(rng):
    """Seeded synthetic 7B-shaped GGUF weights in a Q4_K_M-like mix: Q4_K for
    wq, wk, wo, ffn_gate, ffn_up and the embedding table, Q6_K for wv,
    ffn_down and the output matrix. One layer's host bytes serve every layer
    (each layer gets its own device copy, so every step streams all of them
    from HBM)."""
    from kore_b200.qweights import Q4_K, Q6_K, random_qmat
    E = H * D
    lw = dict(wq=random_qmat(Q4_K, E, E, rng), wk=random_qmat(Q4_K, KVD, E, rng), wv=random_qmat(Q6_K, KVD, E, rng),
              wo=random_qmat(Q4_K, E, E, rng), w_gate=random_qmat(Q4_K, S_FF, E, rng),
              w_up=random_qmat(Q4_K, S_FF, E, rng), w_down=random_qmat(Q6_K, E, S_FF, rng))
    lw.update(bq=rng.standard_normal(E).astype(np.float32) * 0.1, bk=rng.standard_normal(KVD).astype(np.float32) * 0.1,
              bv=rng.standard_normal(KVD).astype(np.float32) * 0.1,
              attn_norm=(1 + 0.1 * rng.standard_normal(E)).astype(np.float32),
              ffn_norm=(1 + 0.1 * rng.standard_normal(E)).astype(np.float32))
    tok = random_qmat(Q4_K, S_VOCAB, E, rng, sigma=1.0)
    out_w = random_qmat(Q6_K, S_VOCAB, E, rng)
    out_norm = (1 + 0.1 * rng.standard_normal(E)).astype(np.float32)
    return lw, tok, out_w, out_norm


def run_step_line(args) -> dict:
    """kore's whole decode step on the device (kore_cuda_decode_step) at the
    headline's shape and position: 7B, 28 layers, KV cache of 32768 seeded
    rows per layer, synthetic Q4_K_M-like weights. One step = one token
    through embedding, 28 layers (RMSNorm, Q8_K, QKV, attention, Wo, residual,
    RMSNorm, gate/up + SwiGLU, down, residual), output norm, logits and
    argmax; the next token is chained on the device. value: tokens/s
    (device-resident, CUDA graph of one step at position POS, events around K
    replays); roofline over weight + KV bytes per step; e2e: the host entry
    point kore_cuda_decode_step (token id in, next token id out) per step."""
    import torch
    import kore_b200 as K
    dev = torch.device("cuda", 0)
    E = H * D
    ctx = K.KoreCuda(L, H, G, D, CTX, device=0)
    stream = torch.cuda.Stream(device=dev)
    ctx.set_stream(stream.cuda_stream)
    rng = np.random.default_rng(81)
    lw, tok, out_w, out_norm = step_model(rng)
    ctx.set_model(S_FF, S_VOCAB, 1e-6, tok, out_norm, out_w, [lw] * L)
    w_bytes = L * sum(lw[k].nbytes for k in ("wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down")) + out_w.nbytes
    with torch.cuda.stream(stream):
        for layer in range(L):
            k, v = layer_rows(torch, dev, layer, POS)
            ctx.append_dev(0, layer, 0, POS, k, v)
            del k, v
        t = torch.tensor([17], dtype=torch.int32, device=dev)
    ctx.sync()

    def step():
        ctx.decode_step_dev(0, t, POS, t)

    warm = max(3, args.warmup)
    with torch.cuda.stream(stream):
        for _ in range(warm):
            step()
    ctx.sync()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    with torch.cuda.stream(stream):
        graph.replay()
    ctx.sync()
    steps = max(20, args.steps // 10)
    clocks = ClockSampler(0)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
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
    # end to end: kore's call, token id in, next token id out
    tok_id = int(t.item())
    for _ in range(3):
        tok_id = ctx.decode_step(0, tok_id, POS)[0]
    n_e2e = max(10, args.e2e_steps // 5)
    t0 = time.perf_counter()
    for _ in range(n_e2e):
        tok_id = ctx.decode_step(0, tok_id, POS)[0]
    e2e_ms = (time.perf_counter() - t0) * 1e3 / n_e2e
    ctx.close()
    kv_bytes = L * layer_bytes(POS)
    step_bytes = kv_bytes + w_bytes
    peaks = load_peaks()
    gbs = step_bytes / (ms * 1e-3) / 1e9
    line = {
        "metric": "decode step tokens/s @7B ctx 32k (whole model on the GPU: 28 layers + logits + argmax)",
        "value": round(1e3 / ms, 2), "unit": "tokens/s", "ms_per_step": round(ms, 4), "steps": steps, "warmup": warm,
        "higher_is_better": True, "dtype": "f32 (Q8_K x Q4_K/Q6_K integer products, fp32 attention)",
        "data": "synthetic (seeded Q4_K_M-like GGUF weights, seeded N(0,1) KV cache)",
        "config": {"workload": f"Qwen2.5-7B-shaped decode step at position {POS}: n_embd 3584, 28Q/4KV, d128, "
                               f"n_ff {S_FF}, vocab {S_VOCAB}, {L} layers",
                   "weights": "Q4_K wq/wk/wo/gate/up/embedding, Q6_K wv/down/output", "weight_bytes_per_step": int(w_bytes),
                   "kv_bytes_per_step": int(kv_bytes), "l2": "8 GB per step > L2, no flush needed"},
        "e2e": {"value": round(1e3 / e2e_ms, 2), "unit": "tokens/s", "ms_per_step": round(e2e_ms, 4),
                "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 260,
                "call": "kore_cuda_decode_step (token id in as an argument; error word + next token id back)"},
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"], "peak_source": peaks["source"],
                     "unit": "GB/s", "frac": round(gbs / peaks["hbm_gbs"], 4),
                     "algorithmic_bytes_per_step": int(step_bytes),
                     "kernels": "embed + 28 x (qmatvec QKV, attn_decode with its split merge, qmatvec Wo, "
                                "qmatvec gate/up, qmatvec down) + qmatvec logits + token"},
        "gpu_launches": steps * (2 + L * (5 + merge_launch()) + 1),
        "clocks": clk,
    }
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = step_cpu_baseline(lw, out_w)
    return line


PM_TOKENS = 2048   # prompt tokens of the whole-model prefill line


def run_prefill_model(args, reuse=None) -> dict:
    """kore's forward_batch() for a whole prompt on the device
    (kore_cuda_prefill): a 2048-token prompt at position 0 through the
    7B-shaped model of the decode-step line (embedding, 28 layers of RMSNorm,
    kore's float batched products with biases / residual adds / SwiGLU, the
    tensor-core prefill attention, then the last token's logits and greedy
    token). value: prompt tokens/s, wall clock around the synchronous call
    (its token ids in, the next token id out). The products are fused
    multiply-add chains on the CUDA cores (kore's order, bit for bit), so the
    roofline is the nominal fp32 CUDA-core peak (no measured one on this
    pool)."""
    import torch
    import kore_b200 as K
    dev = torch.device("cuda", 0)
    ctx = K.KoreCuda(L, H, G, D, PM_TOKENS + 8, device=0)
    rng = np.random.default_rng(81)
    lw, tok, out_w, out_norm = reuse if reuse is not None else step_model(rng)
    ctx.set_model(S_FF, S_VOCAB, 1e-6, tok, out_norm, out_w, [lw] * L)
    toks = np.random.default_rng(83).integers(0, S_VOCAB, PM_TOKENS).astype(np.int32)
    warm = max(2, min(args.warmup, 3))
    for _ in range(warm):
        ctx.prefill_tokens(0, toks, 0)
    steps = 3
    clocks = ClockSampler(0)
    clocks.start()
    torch.cuda.synchronize(dev)
    t_begin = time.time()
    t0 = time.perf_counter()
    for _ in range(steps):
        ctx.prefill_tokens(0, toks, 0)
    ms = (time.perf_counter() - t0) * 1e3 / steps
    t_end = time.time()
    clk = clocks.stop(t_begin, t_end)
    ctx.close()
    E = H * D
    fma = PM_TOKENS * L * (E * (E + 2 * KVD + E) + 3 * S_FF * E)     # the float products
    attn_flop = 4 * D * prefill_pairs(0, PM_TOKENS) * H * L
    tflops = 2 * fma / (ms * 1e-3) / 1e12
    nominal = 148 * 128 * 2 * 1.965e9 / 1e12   # fp32 FMA lanes x 2 x max SM clock
    line = {
        "metric": "whole-model prefill tokens/s @7B (2048-token prompt, 28 layers, kore's float products bit for bit)",
        "value": round(PM_TOKENS / (ms * 1e-3), 1), "unit": "tokens/s", "ms_per_step": round(ms, 2),
        "steps": steps, "warmup": warm, "higher_is_better": True,
        "config": {"workload": f"Qwen2.5-7B-shaped prefill of {PM_TOKENS} tokens at position 0: n_embd 3584, 28Q/4KV, "
                               f"d128, n_ff {S_FF}, vocab {S_VOCAB}, {L} layers (the decode-step line's weights)",
                   "product_fma": int(fma), "attention_flop": int(attn_flop)},
        "e2e": {"value": round(PM_TOKENS / (ms * 1e-3), 1), "unit": "tokens/s", "ms_per_step": round(ms, 2),
                "h2d_bytes_per_step": PM_TOKENS * 4, "d2h_bytes_per_step": 260,
                "note": "the call is synchronous: token ids in, the next token id out; value and e2e are the same call"},
        "roofline": {"bound": "fp32 CUDA cores (products)", "achieved": round(tflops, 1),
                     "peak": round(nominal, 1), "unit": "TFLOP/s", "frac": round(tflops / nominal, 4),
                     "peak_source": "nominal: 148 SMs x 128 fp32 lanes x 2 x 1965 MHz (no measured fp32 peak)",
                     "note": "achieved counts the products' 2 x FMAs only, over the whole call's time"},
        "gpu_launches": steps * (1 + L * 11 + 2),   # per layer: 2 norms, 5 products, append, operand split, attention
        "clocks": clk,
    }
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = prefill_model_cpu_baseline(lw)
    return line


def prefill_model_cpu_baseline(lw) -> dict:
    """kore's own matmul_batch_float (its prefill products) on this host for
    one layer's seven matrices with a 64-token chunk (KORE_BMAX), all host
    threads, scaled to the 2048-token prompt and 28 layers (the attention and
    the rest are left out, so this is an upper bound on kore's speed)."""
    from oracle import oracle as O
    if not O.engine_available():
        return {"value": None, "unavailable": "oracle/_ref/libkore_engine.so not built"}
    cores = len(os.sched_getaffinity(0))
    eng = O.GreedyEngine(1, 512, 4, 2, 512, 32, ctx=8, seed=1, threads=cores)
    E = H * D
    rng = np.random.default_rng(84)
    xe = rng.standard_normal((64, E)).astype(np.float32)
    xf = rng.standard_normal((64, S_FF)).astype(np.float32)
    t = 0.0
    for k in ("wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down"):
        x = xf if k == "w_down" else xe
        best = None
        for _ in range(2):
            t0 = time.perf_counter()
            eng.matmul_batch_ref(lw[k], x)
            dt = time.perf_counter() - t0
            best = dt if best is None else min(best, dt)
        t += best
    ms = t * 1e3 * (PM_TOKENS / 64) * L
    return {"value": round(PM_TOKENS / (ms * 1e-3), 3), "unit": "tokens/s", "cores": cores, "kind": "reference",
            "ms_per_step": round(ms, 1),
            "sample": f"kore's matmul_batch_float of one layer's 7 matrices on a 64-token chunk, {cores} threads, "
                      f"best of 2 each: {t * 1e3:.1f} ms, x {PM_TOKENS // 64} chunks x {L} layers (products only)"}


def step_cpu_baseline(lw, out_w) -> dict:
    """kore's own decode step on this host, composed from its own functions
    (the reference compiled in place): per layer its attention at POS on one
    core (kore's attention is single-threaded) plus its quantize + matvec_mt
    of the layer's seven matrices with all host threads (kore's products are
    threaded), 28 times, plus the output matrix."""
    from oracle import oracle as O
    if not O.ref_available():
        return {"value": None, "unavailable": "oracle/_ref not built"}
    cores = len(os.sched_getaffinity(0))
    rng = np.random.default_rng(82)
    E = H * D
    x = rng.standard_normal(E).astype(np.float32)
    xf = rng.standard_normal(S_FF).astype(np.float32)
    mats = [(lw[k], x) for k in ("wq", "wk", "wv", "wo", "w_gate", "w_up")] + [(lw["w_down"], xf)]
    layer_mv = sum(O.ref_qmatvec_ms(m, v, cores, 3)[0] for m, v in mats)
    out_mv = O.ref_qmatvec_ms(out_w, x, cores, 3)[0]
    e = _ref_engine_with_rows(*[a.astype(np.float32) for a in
                                np.random.default_rng(100).standard_normal((2, POS, KVD), dtype=np.float32)], POS)
    q, k, v = O.seeded_inputs(5, (H * D,), (KVD,), (KVD,))
    t = min(_ref_decode_ms(e, POS, q, k, v) for _ in range(2))
    base = _ref_decode_ms(e, 0, q, k, v, reps=3)
    att = max(t - base, 1e-6)
    ms = L * (att + layer_mv) + out_mv
    return {"value": round(1e3 / ms, 4), "unit": "tokens/s", "cores": cores, "kind": "reference",
            "ms_per_step": round(ms, 1),
            "sample": f"kore's own functions: attention at pos {POS} on 1 core ({att:.1f} ms per layer) + quantize "
                      f"+ matvec_mt of one layer's 7 matrices on {cores} threads ({layer_mv:.1f} ms), x {L} layers, "
                      f"+ the output matrix ({out_mv:.1f} ms); best of 3 each"}


# ---------------------------------------------------------------- config 5: batched decode

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

    warm = max(3, args.warmup)
    with torch.cuda.stream(stream):
        for _ in range(warm):
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
    clocks = ClockSampler(dev.index)
    clocks.start()
    barrier()
    t_begin = time.time()
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(steps):
            graph.replay()
        e1.record(stream)
    e1.synchronize()
    t_end = time.time()
    clk = clocks.stop(t_begin, t_end)
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
        "value": round(gbs, 1), "unit": "GB/s", "n_gpus": world, "steps": steps, "warmup": warm,
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
        "clocks": clk,
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

    warm = 3
    with torch.cuda.stream(stream):
        for _ in range(warm):
            step()
    ctx.sync()
    steps = args.prefill_steps
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(dev.index)
    clocks.start()
    t_begin = time.time()
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(steps):
            step()
        e1.record(stream)
    e1.synchronize()
    t_end = time.time()
    clk = clocks.stop(t_begin, t_end)
    ctx.sync()
    ms = e0.elapsed_time(e1) / steps
    flops = 4 * D * prefill_pairs(P0, N) * H * LP
    tflops = flops / (ms * 1e-3) / 1e12
    ctx.close()
    # the tensor pipe runs three bf16 MMAs per fp32-accurate product
    peak_eq = peaks["bf16_tflops"] / 3
    return {"metric": "prefill attn TFLOP/s (7B, 2048-token chunk onto 4096, 28 layers)",
            "value": round(tflops, 1), "unit": "TFLOP/s", "ms_per_step": round(ms, 4), "steps": steps,
            "warmup": warm, "layers": LP, "flop_per_step": flops,
            "roofline": {"bound": "tensor", "achieved": round(tflops, 1), "peak": round(peak_eq, 1),
                         "unit": "TFLOP/s", "frac": round(tflops / peak_eq, 4), "peak_source": peaks["source"],
                         "peak_note": "measured bf16 dense peak / 3: each fp32-accurate product is three bf16 "
                                      "MMAs (hi*hi + hi*mid + mid*hi)",
                         "frac_of_bf16_peak": round(tflops / peaks["bf16_tflops"], 4),
                         "bf16_peak": peaks["bf16_tflops"]},
            "kernels": "kv_append_kernel + kv_split_kernel + prefill_kernel (tcgen05, TMEM)",
            "clocks": clk}


def load_peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            j = json.load(f)
        return {"hbm_gbs": float(j["hbm_gbs"]), "bf16_tflops": float(j["bf16_tflops"]), "source": "measured"}
    except (OSError, KeyError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def merge_launch(world: int = 1) -> int:
    """Launches a single-query decode adds for its split merge (world == 1) or
    its peer exchange (world > 1): 0 when they run in the decode's own launch
    (the default), 1 when KORE_CUDA_FUSED_MERGE / KORE_CUDA_FUSED_EXCHANGE=0."""
    var = "KORE_CUDA_FUSED_MERGE" if world == 1 else "KORE_CUDA_FUSED_EXCHANGE"
    return 0 if os.environ.get(var, "1") != "0" else 1


def load_traffic():
    """DRAM bytes per decode launch from the committed ncu summary, if any."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(p) as f:
            return json.load(f).get("attn_decode_cfg4_bytes_per_launch")
    except (OSError, ValueError):
        return None


# ---------------------------------------------------------------- CPU legs (the reference compiled in place)

def _ref_engine_with_rows(k_rows: np.ndarray, v_rows: np.ndarray, pos: int, threads: int = 1):
    from oracle import oracle as O
    e = O.RefLayer(H, G, D, pos + 1, threads=threads)
    for p0 in range(0, pos, 4096):
        e.fill(p0, k_rows[p0:p0 + 4096], v_rows[p0:p0 + 4096])
    return e


def _ref_decode_ms(e, pos: int, q, k, v, reps: int = 1) -> float:
    t0 = time.perf_counter()
    for _ in range(reps):
        e.decode(pos, q, k, v)
    return (time.perf_counter() - t0) * 1e3 / reps


def cpu_baseline_sample(pos: int, gpu_layer0, q0, k0, v0):
    """kore's own decode attention (forward() of the compiled reference) on 1
    core, one layer at `pos` over the same cache rows and q/k/v as the GPU's
    layer 0, minus the same forward() at position 0 (embedding, norms and
    zero-weight projections, i.e. everything that is not attention). Its
    output is also the N = 1 parity check of the GPU's layer 0. Returns
    (cpu_baseline, parity or None)."""
    from oracle import oracle as O
    if not O.ref_available():
        return {"value": None, "unavailable": "oracle/_ref not built"}, None
    import torch
    dev = torch.device("cuda", 0)
    kr, vr = layer_rows(torch, dev, 0, pos)
    e = _ref_engine_with_rows(kr.cpu().numpy(), vr.cpu().numpy(), pos)
    del kr, vr
    ref = e.decode(pos, q0, k0, v0)   # before any forward() at position 0, which rewrites row 0
    t = min(_ref_decode_ms(e, pos, q0, k0, v0) for _ in range(3))
    base = _ref_decode_ms(e, 0, q0, k0, v0, reps=3)
    att = max(t - base, 1e-6)
    cb = {"value": round(layer_bytes(pos) / (att * 1e-3) / 1e9, 3), "unit": "GB/s", "cores": 1,
          "kind": "reference", "attention_ms": round(att, 3),
          "sample": f"1 of 28 layers, decode at pos {pos}, kore forward() best of 3 = {t:.1f} ms "
                    f"minus forward() at pos 0 = {base:.1f} ms; attention {att:.1f} ms"}
    par = parity_entry(gpu_layer0, ref.reshape(-1), "kore's own forward() (oracle/_ref) on the same cache rows "
                       "and q/k/v as the GPU's layer 0")
    return cb, par


def run_reference(args, rank: int, world: int) -> dict | None:
    """The reference arm: kore's own CPU attention for the headline workload.
    Each step is a full 28-layer decode at POS: 28 kore forward() calls, one
    per layer, fanned over the host's cores (kore's attention is
    single-threaded, so one forward() per core is all the parallelism its code
    has), minus the non-attention part of each forward()."""
    if rank != 0:
        return None
    from oracle import oracle as O
    if not O.ref_available():
        return {"impl": "reference", "unavailable": "oracle/_ref/libkore_ref.so not built (needs the reference sources)"}
    cores = len(os.sched_getaffinity(0))
    T = max(1, min(cores, L))
    engines = []
    for i in range(T):
        g = np.random.default_rng(100 + i)
        rows_k = g.standard_normal((POS, KVD), dtype=np.float32)
        rows_v = g.standard_normal((POS, KVD), dtype=np.float32)
        engines.append(_ref_engine_with_rows(rows_k, rows_v, POS))
        del rows_k, rows_v
    q, k, v = O.seeded_inputs(5, (H * D,), (KVD,), (KVD,))
    t1 = min(_ref_decode_ms(engines[0], POS, q, k, v) for _ in range(2))
    base = _ref_decode_ms(engines[0], 0, q, k, v, reps=3)
    one_core_att = max(t1 - base, 1e-6)
    per_thread = (L + T - 1) // T

    def worker(t):
        for layer in range(t, L, T):
            engines[t].decode(POS, q, k, v)

    def one_step():
        ths = [threading.Thread(target=worker, args=(t,)) for t in range(T)]
        t0 = time.perf_counter()
        for th in ths:
            th.start()
        for th in ths:
            th.join()
        return (time.perf_counter() - t0) * 1e3

    budget_s = 240.0
    first = one_step()
    steps = max(1, min(args.steps, int(budget_s * 1e3 / max(first, 1.0)) - args.warmup))
    warm = args.warmup
    for _ in range(max(0, warm - 1)):
        one_step()
    times = [one_step() for _ in range(steps)]
    ms = sum(times) / len(times)
    att_ms = max(ms - per_thread * base, 1e-6)   # each thread ran per_thread non-attention parts too
    step_bytes = L * layer_bytes(POS)
    v_gbs = step_bytes / (att_ms * 1e-3) / 1e9
    one_gbs = layer_bytes(POS) / (one_core_att * 1e-3) / 1e9
    return {
        "impl": "reference", "metric": f"decode attn HBM GB/s @7B ctx {POS // 1024}k ({L} layers, 28Q/4KV, d128, fp32 KV)",
        "value": round(v_gbs, 3), "unit": "GB/s", "n_gpus": world, "steps": steps, "warmup": warm,
        "steps_requested": args.steps, "ms_per_step": round(att_ms, 3), "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1))", "config": cfg4_config(world),
        "readings": {
            "i_reference_as_is_1_core": {"value": round(one_gbs, 3), "unit": "GB/s",
                                         "ms_per_step": round(L * one_core_att, 1),
                                         "note": "kore's attention runs on one core whatever --threads is: "
                                                 f"{L} layers x {one_core_att:.1f} ms"},
            "ii_layers_fanned_over_cores": {"value": round(v_gbs, 3), "unit": "GB/s", "cores": T,
                                            "ms_per_step": round(att_ms, 1),
                                            "note": "the line's value: one kore forward() per core at a time"}},
        "cpu_baseline": {"value": round(v_gbs, 3), "unit": "GB/s", "cores": T, "kind": "reference",
                         "sample": f"each step: all {L} layers decoded at pos {POS}, one kore forward() per layer, "
                                   f"{T} at a time (one per core), minus {per_thread} x forward() at pos 0 "
                                   f"({base:.1f} ms) per thread; {steps} timed steps after {warm} warm-up"},
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
    if args.step_only:
        print(json.dumps(run_step_line(args)), flush=True)
        return
    if args.prefill_model_only:
        print(json.dumps(run_prefill_model(args)), flush=True)
        return
    ok = True
    try:
        line = run_decode(args, rank, world, dist, POS, L, args.steps, args.e2e_steps, want_block=True)
        if not args.no_batched:
            batched = run_batched(args, rank, world, dist, load_peaks())
            if line is not None:
                line["batched"] = batched
        if line is not None and world == 1:
            import torch
            if not args.no_cfg12:
                line["cfg2"] = run_decode(args, 0, 1, None, 8192, 28, max(200, args.steps), max(10, args.e2e_steps),
                                          want_block=False)
                line["cfg1"] = run_cfg1(args)
            if not args.no_prefill:
                line["prefill"] = run_prefill(args, torch.device("cuda", 0), load_peaks())
            if not args.no_step:
                line["decode_step"] = run_step_line(args)
                line["prefill_model"] = run_prefill_model(args)
        if line is not None:
            ok = all(x.get("parity", {}).get("ok", True) for x in (line, line.get("cfg2") or {}))
            print(json.dumps(line), flush=True)
    finally:
        if dist is not None:
            dist.destroy_process_group()
    if not ok:
        print("bench: parity check failed (see the line's parity object)", file=sys.stderr, flush=True)
        sys.exit(3)


if __name__ == "__main__":
    main()
