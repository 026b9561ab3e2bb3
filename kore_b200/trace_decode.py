"""Phase trace of the single-sequence decode (config 4 shape by default).

Runs graph-replayed 28-layer decode steps through the trace build of the
library (``python -m kore_b200.build --trace``: every decode, split-merge and
merge CTA stamps %globaltimer at fixed points) and prints, per layer launch,
where the time goes:

  start      first decode CTA entry of the launch (t = 0)
  released   dependency wait returned (first / median / last CTA)
  staged     q, RoPE row and new token staged (median)
  tiles      the CTA's last tile consumed (first / median / last)
  end        the CTA's partial written (first / median / last)
  merge      merge CTAs: entry, splits seen (fused launch), end (last)
  period     to the next launch's first decode CTA entry

With --step it traces the whole decode step instead (kore_cuda_decode_step_dev
at the 7B shape, synthetic weights): the product CTAs stamp entry, dependency
release, Q8_K input built, first weights landed and end too, and the table
gives, per launch role (qkv, attn, wo, gate_up, down, output), the mean phases
from the launch's first CTA entry and the gap from the previous launch's last
CTA end to this launch's median release.

Usage (on a GPU machine; the trace library is built beforehand):
    python -m kore_b200.trace_decode [--layers 28] [--pos 32768] [--steps 3] [--step]
Environment switches of the library (KORE_CUDA_FUSED_MERGE=0, ...) apply as
usual. The numbers are for comparing phases; a trace build is not timed for
throughput.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

REC = np.dtype([("t", "<u8", 5), ("blk", "<u4"), ("sm", "<u4"), ("kind", "<u4"), ("tag", "<u4"), ("pad2", "<u8")])
assert REC.itemsize == 64


def read_trace(lib) -> np.ndarray:
    buf = np.zeros(1 << 16, REC)
    n = ctypes.c_int(0)
    rc = lib.kore_trace_read(buf.ctypes.data_as(ctypes.c_void_p), len(buf), ctypes.byref(n))
    if rc:
        raise RuntimeError(f"kore_trace_read failed ({rc})")
    return buf[: n.value]


def launches(recs: np.ndarray) -> list[tuple[np.ndarray, np.ndarray]]:
    """Splits the records (in claim order) into launches: a run of decode CTAs
    followed by the run of merge CTAs that belongs to it."""
    out, dec, mer = [], [], []
    for r in recs:
        if r["kind"] == 0:
            if mer:
                out.append((np.array(dec, REC), np.array(mer, REC)))
                dec, mer = [], []
            dec.append(r)
        else:
            mer.append(r)
    if dec:
        out.append((np.array(dec, REC), np.array(mer, REC)))
    return out


def phase_table(ls: list[tuple[np.ndarray, np.ndarray]]) -> dict:
    rows = []
    for i, (dec, mer) in enumerate(ls):
        t0 = int(dec["t"][:, 0].min())
        us = lambda x: (np.asarray(x, np.float64) - t0) / 1e3  # noqa: E731
        done = dec[dec["t"][:, 4] > 0]   # CTAs past their split count return early
        row = {
            "decode_ctas": len(dec),
            "entry_last": float(us(dec["t"][:, 0].max())),
            "released": [float(x) for x in np.percentile(us(done["t"][:, 1]), [0, 50, 100])],
            "staged_med": float(np.median(us(done["t"][:, 2]))),
            "tiles": [float(x) for x in np.percentile(us(done["t"][:, 3]), [0, 50, 100])],
            "end": [float(x) for x in np.percentile(us(done["t"][:, 4]), [0, 50, 100])],
        }
        if len(mer):
            row["merge_kind"] = int(mer["kind"][0])
            row["merge_entry_first"] = float(us(mer["t"][:, 0].min()))
            row["merge_released_last"] = float(us(mer["t"][:, 1].max()))
            if mer["kind"][0] == 2:
                row["merge_seen_last"] = float(us(mer["t"][:, 2].max()))
            row["merge_end_last"] = float(us(mer["t"][:, 4].max()))
        if i + 1 < len(ls):
            row["period"] = float(us(ls[i + 1][0]["t"][:, 0].min()))
        rows.append(row)
    body = [r for r in rows if "period" in r][1:]   # steady state: not the first or last launch
    keys = ["entry_last", "staged_med", "merge_entry_first", "merge_released_last", "merge_seen_last",
            "merge_end_last", "period"]
    mean = {k: float(np.mean([r[k] for r in body if k in r])) for k in keys if any(k in r for r in body)}
    for k in ("released", "tiles", "end"):
        mean[k] = [float(np.mean([r[k][j] for r in body])) for j in range(3)]
    return {"launches": len(rows), "steady_launches": len(body), "mean_us": mean, "per_launch": rows}


# ---------------------------------------------------------------- the whole decode step

# product launches by their shape tag (qmatvec kinds 3 and 4): out_mode, n_seg
OUT_STORE, OUT_RESIDUAL, OUT_SWIGLU, OUT_ARGMAX = 0, 1, 2, 3


def product_role(rec, n_embd: int) -> str:
    out_mode = int(rec["pad2"] >> 32) & 0xFF
    n_seg = int(rec["pad2"] >> 40) & 0xFF
    cols = int(rec["pad2"] & 0xFFFFFFFF)
    if out_mode == OUT_SWIGLU:
        return "gate_up"
    if out_mode == OUT_ARGMAX:
        return "output"
    if out_mode == OUT_RESIDUAL:
        return "wo" if cols == n_embd else "down"
    return "qkv" if n_seg == 3 else f"store{n_seg}"


def step_launches(recs: np.ndarray, n_embd: int) -> list[dict]:
    """Every launch of the traced steps in start order: the decode launches
    (decode CTAs with their merge CTAs) and the product launches (a run of
    records of one shape tag; consecutive product launches of a step always
    differ in shape)."""
    dec = recs[(recs["kind"] == 0) | (recs["kind"] == 1) | (recs["kind"] == 2)]
    prod = recs[(recs["kind"] == 3) | (recs["kind"] == 4)]
    out = []
    for d, m in launches(dec):
        done = d[d["t"][:, 4] > 0]
        out.append({"role": "attn", "t0": int(d["t"][:, 0].min()), "recs": done, "merge": m})
    run = []
    for r in prod:
        if run and (r["kind"], r["tag"], r["pad2"]) != (run[-1]["kind"], run[-1]["tag"], run[-1]["pad2"]):
            out.append({"role": product_role(run[0], n_embd), "t0": int(min(x["t"][0] for x in run)),
                        "recs": np.array(run, REC)})
            run = []
        run.append(r)
    if run:
        out.append({"role": product_role(run[0], n_embd), "t0": int(min(x["t"][0] for x in run)),
                    "recs": np.array(run, REC)})
    out.sort(key=lambda x: x["t0"])
    return out


def step_table(ls: list[dict]) -> dict:
    """Per launch role, the mean over the steady launches (not the first or
    last of the trace) of its phases in us from its first CTA entry, and the
    dependency gap: the previous launch's last CTA end to this launch's
    median dependency release."""
    rows = []
    for i, l in enumerate(ls):
        r = l["recs"]
        t0 = l["t0"]
        us = lambda x: (np.asarray(x, np.float64) - t0) / 1e3  # noqa: E731
        row = {"role": l["role"], "ctas": len(r),
               "entry_last": float(us(r["t"][:, 0].max())),
               "released_med": float(np.median(us(r["t"][:, 1]))),
               "end_med": float(np.median(us(r["t"][:, 4]))),
               "end_last": float(us(r["t"][:, 4].max()))}
        if l["role"] != "attn":
            row["built_med"] = float(np.median(us(r["t"][:, 2])))
            landed = r["t"][:, 3][r["t"][:, 3] > 0]
            if len(landed):
                row["landed_med"] = float(np.median(us(landed)))
        else:
            row["staged_med"] = float(np.median(us(r["t"][:, 2])))
            if len(l["merge"]):
                row["end_last"] = max(row["end_last"], float(us(l["merge"]["t"][:, 4].max())))
        if i > 0:
            prev_end = ls[i - 1]["t0"] + 1e3 * rows[-1]["end_last"]
            row["gap_from_prev_end"] = float((t0 + 1e3 * row["released_med"] - prev_end) / 1e3)
        if i + 1 < len(ls):
            row["period"] = float(us(ls[i + 1]["t0"]))
        rows.append(row)
    body = rows[1:-1]
    roles = []
    for r in body:
        if r["role"] not in roles:
            roles.append(r["role"])
    mean = {}
    for role in roles:
        rs = [r for r in body if r["role"] == role and "period" in r]
        keys = sorted({k for r in rs for k in r if k not in ("role", "ctas")})
        mean[role] = {k: round(float(np.mean([r[k] for r in rs if k in r])), 3) for k in keys}
        mean[role]["launches"] = len(rs)
    return {"launches": len(rows), "mean_us": mean, "per_launch": rows}


def run_step(args, lib) -> dict:
    """Traces graph-replayed whole decode steps (kore_cuda_decode_step_dev)
    at the 7B shape with synthetic Q4_K_M-like weights (Q4_K wq/wk/wo/gate/up/
    embedding, Q6_K wv/down/output) and a seeded cache of args.pos rows."""
    import torch
    import kore_b200 as K
    from kore_b200.qweights import Q4_K, Q6_K, random_qmat

    H, G, D, FF, VOCAB = 28, 4, 128, 18944, 152064
    E, KVD = H * D, G * D
    rng = np.random.default_rng(81)
    lw = dict(wq=random_qmat(Q4_K, E, E, rng), wk=random_qmat(Q4_K, KVD, E, rng), wv=random_qmat(Q6_K, KVD, E, rng),
              wo=random_qmat(Q4_K, E, E, rng), w_gate=random_qmat(Q4_K, FF, E, rng),
              w_up=random_qmat(Q4_K, FF, E, rng), w_down=random_qmat(Q6_K, E, FF, rng),
              bq=rng.standard_normal(E).astype(np.float32) * 0.1, bk=rng.standard_normal(KVD).astype(np.float32) * 0.1,
              bv=rng.standard_normal(KVD).astype(np.float32) * 0.1,
              attn_norm=(1 + 0.1 * rng.standard_normal(E)).astype(np.float32),
              ffn_norm=(1 + 0.1 * rng.standard_normal(E)).astype(np.float32))
    tok = random_qmat(Q4_K, VOCAB, E, rng, sigma=1.0)
    out_w = random_qmat(Q6_K, VOCAB, E, rng)
    out_norm = (1 + 0.1 * rng.standard_normal(E)).astype(np.float32)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    ctx = K.KoreCuda(args.layers, H, G, D, args.pos + 1, device=0)
    stream = torch.cuda.Stream(device=dev)
    ctx.set_stream(stream.cuda_stream)
    ctx.set_model(FF, VOCAB, 1e-6, tok, out_norm, out_w, [lw] * args.layers)
    gen = torch.Generator(device=dev)
    with torch.cuda.stream(stream):
        for layer in range(args.layers):
            gen.manual_seed(1000 + layer)
            k = torch.randn(args.pos, KVD, device=dev, generator=gen)
            v = torch.randn(args.pos, KVD, device=dev, generator=gen)
            ctx.append_dev(0, layer, 0, args.pos, k, v)
            del k, v
        t = torch.tensor([17], dtype=torch.int32, device=dev)
    ctx.sync()

    def step():
        ctx.decode_step_dev(0, t, args.pos, t)

    recs = _trace_graph(args, lib, stream, step)
    ctx.close()
    table = step_table(step_launches(recs, E))
    table["config"] = {"layers": args.layers, "pos": args.pos, "steps": args.steps, "mode": "step"}
    return table, recs


def _trace_graph(args, lib, stream, step) -> np.ndarray:
    import torch
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    with torch.cuda.stream(stream):
        graph.replay()
    torch.cuda.synchronize()
    if lib.kore_trace_reset():
        raise RuntimeError("kore_trace_reset failed")
    with torch.cuda.stream(stream):
        for _ in range(args.steps):
            graph.replay()
    torch.cuda.synchronize()
    recs = read_trace(lib)
    del graph
    return recs


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=28)
    ap.add_argument("--pos", type=int, default=32768)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--per-launch", action="store_true", help="print every launch's row")
    ap.add_argument("--dump", default="", help="also save the raw records (numpy .npy) to this path")
    ap.add_argument("--between-mb", type=int, default=0,
                    help="attention alone: a torch read of this many MB (one buffer) between the layers' decodes, "
                         "so that each decode follows another kernel, as in the whole step")
    ap.add_argument("--step", action="store_true",
                    help="trace the whole decode step (products, attention, merge) instead of attention alone")
    args = ap.parse_args()

    import torch
    import kore_b200 as K
    from kore_b200.build import TRACE_LIB

    if not os.path.exists(TRACE_LIB):
        raise SystemExit(f"{TRACE_LIB} is missing: build it with `python -m kore_b200.build --trace`")
    lib = K.load_library(TRACE_LIB)
    lib.kore_trace_read.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_int)]
    lib.kore_trace_reset.argtypes = []

    if args.step:
        table, recs = run_step(args, lib)
        if args.dump:
            np.save(args.dump, recs)
        if not args.per_launch:
            table.pop("per_launch")
        print(json.dumps(table))
        return

    H, G, D = 28, 4, 128
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    ctx = K.KoreCuda(args.layers, H, G, D, args.pos + 1, device=0)
    stream = torch.cuda.Stream(device=dev)
    ctx.set_stream(stream.cuda_stream)
    gen = torch.Generator(device=dev)
    with torch.cuda.stream(stream):
        for layer in range(args.layers):
            gen.manual_seed(1000 + layer)
            k = torch.randn(args.pos, G * D, device=dev, generator=gen)
            v = torch.randn(args.pos, G * D, device=dev, generator=gen)
            ctx.append_dev(0, layer, 0, args.pos, k, v)
            del k, v
        gen.manual_seed(7)
        q = torch.randn(args.layers, H * D, device=dev, generator=gen)
        kn = torch.randn(args.layers, G * D, device=dev, generator=gen)
        vn = torch.randn(args.layers, G * D, device=dev, generator=gen)
        out = torch.empty(args.layers, H * D, device=dev)
        between = torch.ones(args.between_mb << 18, device=dev) if args.between_mb > 0 else None
        sums = torch.zeros(args.layers, device=dev)
    ctx.sync()

    def step():
        for layer in range(args.layers):
            ctx.decode_dev(0, layer, args.pos, q[layer], kn[layer], vn[layer], out[layer])
            if between is not None:
                torch.sum(between, dim=0, out=sums[layer])

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
    ctx.sync()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    with torch.cuda.stream(stream):
        graph.replay()
    torch.cuda.synchronize()
    if lib.kore_trace_reset():
        raise RuntimeError("kore_trace_reset failed")
    with torch.cuda.stream(stream):
        for _ in range(args.steps):
            graph.replay()
    torch.cuda.synchronize()
    recs = read_trace(lib)
    if args.dump:
        np.save(args.dump, recs)
    del graph
    ctx.close()
    table = phase_table(launches(recs))
    if not args.per_launch:
        table.pop("per_launch")
    table["config"] = {"layers": args.layers, "pos": args.pos, "steps": args.steps, "between_mb": args.between_mb,
                       "fused_merge": os.environ.get("KORE_CUDA_FUSED_MERGE", "1")}
    print(json.dumps(table))


if __name__ == "__main__":
    main()
