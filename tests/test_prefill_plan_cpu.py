"""The prefill work list (kore::prefill_plan, attn_prefill.cu), host logic, CPU only.

A small C++ driver linked against the built library prints the plan of a
chunk shape; the test checks what the prefill kernel relies on: every
(query head, 128-row query tile) is covered exactly once, either whole or as
two halves of one split slot; the halves partition the tile's key tiles, the
first ending no later than the tile's first masked key tile (so it needs no
mask) and each half having at least 4 key tiles; split slots are numbered
0..slots-1 with parts 0 and 1 each used once.
"""
import os
import shutil
import subprocess

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(REPO, "kore_b200")
CUDA_INC = "/usr/local/cuda/include"

DRIVER = r"""
#include <cstdio>
#include <cstdlib>
#include <vector>
#include <vector_types.h>
namespace kore { int prefill_plan(int pos0, int n, int H, int num_sms, std::vector<int4> &items); }
int main(int argc, char **argv) {
    const int pos0 = atoi(argv[1]), n = atoi(argv[2]), H = atoi(argv[3]), sms = atoi(argv[4]);
    std::vector<int4> items;
    const int slots = kore::prefill_plan(pos0, n, H, sms, items);
    printf("%d %zu\n", slots, items.size());
    for (const int4 &it : items) printf("%d %d %d %d\n", it.x, it.y, it.z, it.w);
    return 0;
}
"""


@pytest.fixture(scope="module")
def driver(tmp_path_factory):
    if not os.path.exists(os.path.join(LIBDIR, "libkore_cuda.so")):
        pytest.skip("kore_b200/libkore_cuda.so not built")
    if not shutil.which("g++") or not os.path.exists(os.path.join(CUDA_INC, "vector_types.h")):
        pytest.skip("g++ or the CUDA headers are missing")
    d = tmp_path_factory.mktemp("plan")
    src, exe = d / "plan.cpp", d / "plan"
    src.write_text(DRIVER)
    subprocess.run(["g++", "-std=c++17", "-O1", "-I", CUDA_INC, str(src), "-o", str(exe), "-L", LIBDIR,
                    "-lkore_cuda", f"-Wl,-rpath,{LIBDIR}"], check=True)
    return str(exe)


def plan(driver, pos0, n, H, sms=148):
    out = subprocess.run([driver, str(pos0), str(n), str(H), str(sms)], check=True, capture_output=True,
                         text=True).stdout.split("\n")
    slots, count = map(int, out[0].split())
    items = [tuple(map(int, line.split())) for line in out[1:1 + count]]
    assert len(items) == count
    return slots, items


@pytest.mark.parametrize("pos0,n,H,sms", [
    (4096, 2048, 28, 148),    # config 3: the heaviest tiles are split
    (0, 2048, 28, 148),
    (0, 128, 28, 148),
    (100, 300, 14, 148),
    (0, 1, 4, 148),
    (8000, 64, 16, 148),
    (30000, 2048, 28, 148),
    (5, 7, 2, 148),
    (4096, 2048, 28, 132),    # another SM count
    (12000, 4096, 40, 148),
])
def test_plan_covers_every_tile_once_and_splits_soundly(driver, pos0, n, H, sms):
    slots, items = plan(driver, pos0, n, H, sms)
    q_tiles = (n + 127) // 128
    whole, halves = {}, {}
    for h, qt, tt, w in items:
        assert 0 <= h < H and 0 <= qt < q_tiles
        t0, t1 = tt & 0xFFFF, tt >> 16
        z0 = qt * 128
        rows = min(128, n - z0)
        nt = (pos0 + z0 + rows - 1) // 128 + 1      # key tiles the tile's last row reaches
        fm = (pos0 + z0) // 128                      # first key tile that needs the causal mask
        if w < 0:
            assert (h, qt) not in whole and (h, qt) not in halves
            assert (t0, t1) == (0, nt)
            whole[(h, qt)] = True
        else:
            slot, part = w >> 1, w & 1
            assert 0 <= slot < slots
            halves.setdefault((h, qt), {})[part] = (t0, t1, slot, nt, fm)
    for key, parts in halves.items():
        assert key not in whole
        assert sorted(parts) == [0, 1], key
        (a0, a1, s0, nt, fm), (b0, b1, s1, _, _) = parts[0], parts[1]
        assert s0 == s1
        assert a0 == 0 and a1 == b0 and b1 == nt      # the halves partition [0, nt)
        assert a1 <= fm                               # the first half is unmasked
        assert a1 >= 4 and nt - a1 >= 4
    assert len(whole) + len(halves) == H * q_tiles
    assert len(items) == H * q_tiles + slots
    assert sorted(p[0][2] for p in halves.values()) == list(range(slots))


def test_config3_plan_splits_the_heaviest_tiles(driver):
    slots, items = plan(driver, 4096, 2048, 28)
    assert slots > 0
    # every split tile is at least as long as every whole one
    lens = {}
    for h, qt, tt, w in items:
        nt = (4096 + qt * 128 + 127) // 128 + 1
        lens.setdefault(w >= 0, set()).add(nt)
    assert min(lens[True]) >= max(lens[False])


def test_small_chunks_are_not_split(driver):
    for pos0, n in ((0, 128), (0, 2048), (100, 300)):
        slots, _ = plan(driver, pos0, n, 28)
        assert slots == 0
