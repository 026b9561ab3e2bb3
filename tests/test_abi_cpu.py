"""The C-ABI library loads and exports every entry point include/*.h declares;
creating a context without a usable GPU fails cleanly with a message.
CPU only: no kernel runs here."""
import ctypes
import os
import subprocess

import pytest

import kore_b200 as K


def test_header_declares_the_boundary():
    names = K.declared_symbols()
    for must in ("kore_cuda_create", "kore_cuda_destroy", "kore_cuda_kv_append", "kore_cuda_attn_prefill",
                 "kore_cuda_attn_decode", "kore_cuda_attn_decode_batch", "kore_cuda_last_error"):
        assert must in names


def test_library_exports_every_declared_symbol():
    lib = K.load_library()
    missing = [n for n in K.declared_symbols() if not hasattr(lib, n)]
    assert not missing, f"declared in include/ but not exported: {missing}"


def test_exports_are_c_symbols():
    out = subprocess.run(["nm", "-D", "--defined-only", K.LIB], capture_output=True, text=True, check=True).stdout
    exported = {l.split()[-1] for l in out.splitlines() if " T " in l}
    for n in K.declared_symbols():
        assert n in exported, n   # unmangled: callable from C, cgo, JNI or ctypes


def test_cfg_default_fills_kore_defaults():
    lib = K.load_library()
    cfg = K._Cfg()
    lib.kore_cuda_cfg_default(ctypes.byref(cfg), 28, 28, 4, 128, 8193)
    assert (cfg.n_layer, cfg.n_head, cfg.n_head_kv, cfg.head_dim, cfg.ctx_max) == (28, 28, 4, 128, 8193)
    assert cfg.page_tokens == 256 and cfg.max_seqs == 1 and abs(cfg.rope_base - 1e6) < 1
    assert cfg.shard_count == 1 and cfg.shard_rank == 0 and not cfg.inv_freq


@pytest.mark.parametrize("kw,code", [
    (dict(n_head=28, n_head_kv=5), -1),       # H % G != 0
    (dict(n_head=36, n_head_kv=4), -1),       # n_rep 9 > 8
    (dict(head_dim=96), -1),                  # unsupported head_dim
    (dict(page_tokens=100), -1),              # page not a multiple of 64
])
def test_create_rejects_bad_geometry_before_touching_a_gpu(kw, code):
    args = dict(n_layer=2, n_head=28, n_head_kv=4, head_dim=128, ctx_max=64)
    page = kw.pop("page_tokens", 256)
    args.update(kw)
    with pytest.raises(K.KoreCudaError) as e:
        K.KoreCuda(args["n_layer"], args["n_head"], args["n_head_kv"], args["head_dim"], args["ctx_max"],
                   page_tokens=page)
    assert e.value.code == code
    assert str(e.value)


@pytest.mark.skipif(os.environ.get("CUDA_VISIBLE_DEVICES") is None and
                    os.path.exists("/dev/nvidia0"), reason="a GPU is present")
def test_create_without_gpu_reports_error_instead_of_aborting():
    with pytest.raises(K.KoreCudaError) as e:
        K.KoreCuda(2, 28, 4, 128, 64)
    assert e.value.code == -4 and "device" in str(e.value).lower()


def test_c_call_binds_the_context_and_raises_on_error():
    """KoreCuda.c_call (the raw-pointer form kore's own calls take, used by the
    bench's host-buffer timings) passes the context handle first, the
    arguments unchanged, and turns a non-zero return into KoreCudaError."""
    calls = []

    class FakeLib:
        def kore_cuda_x(self, h, *a):
            calls.append((h,) + a)
            return 0 if a[0] >= 0 else 22

        def kore_cuda_last_error(self, h):
            return b"bad argument"

    c = object.__new__(K.KoreCuda)
    c._L, c._h = FakeLib(), "ctx"
    f = c.c_call("kore_cuda_x")
    f(1, 2, 0x1000)
    assert calls == [("ctx", 1, 2, 0x1000)]
    with pytest.raises(K.KoreCudaError, match="bad argument"):
        f(-1)
    c._h = None   # nothing to close
