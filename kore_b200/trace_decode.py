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

Usage (on a GPU machine; the trace library is built beforehand):
    python -m kore_b200.trace_decode [--layers 28] [--pos 32768] [--steps 3]
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

REC = np.dtype([("t", "<u8", 5), ("blk", "<u4"), ("sm", "<u4"), ("kind", "<u4"), ("pad", "<u4"), ("pad2", "<u8")])
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


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=28)
    ap.add_argument("--pos", type=int, default=32768)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--per-launch", action="store_true", help="print every launch's row")
    ap.add_argument("--dump", default="", help="also save the raw records (numpy .npy) to this path")
    args = ap.parse_args()

    import torch
    import kore_b200 as K
    from kore_b200.build import TRACE_LIB

    if not os.path.exists(TRACE_LIB):
        raise SystemExit(f"{TRACE_LIB} is missing: build it with `python -m kore_b200.build --trace`")
    lib = K.load_library(TRACE_LIB)
    lib.kore_trace_read.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_int)]
    lib.kore_trace_reset.argtypes = []

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
    ctx.sync()

    def step():
        for layer in range(args.layers):
            ctx.decode_dev(0, layer, args.pos, q[layer], kn[layer], vn[layer], out[layer])

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
    table["config"] = {"layers": args.layers, "pos": args.pos, "steps": args.steps,
                       "fused_merge": os.environ.get("KORE_CUDA_FUSED_MERGE", "1")}
    print(json.dumps(table))


if __name__ == "__main__":
    main()
