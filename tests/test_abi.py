"""The C-ABI library: it loads, exports every symbol include/*.h declares, and
its host-side argument checks behave as the reference's (no GPU needed)."""
import ctypes as C
import os
import re
import shutil
import subprocess

import numpy as np
import pytest

import build as mvbuild
import cases

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def lib():
    mvbuild.build()
    import mvllm_moe
    return mvllm_moe


def header_symbols():
    with open(os.path.join(ROOT, "include", "mvllm_moe.h")) as f:
        text = f.read()
    return sorted(set(re.findall(r"MVLLM_API [^;(]*?\b(mvllm_\w+)\(", text)))


def test_exports_every_declared_symbol(lib):
    declared = header_symbols()
    assert len(declared) >= 20
    assert set(declared) == set(lib.C_SYMBOLS)
    L = C.CDLL(lib.LIB_PATH)
    for name in declared:
        assert hasattr(L, name), name


def test_cpp_adapter_symbol_matches_reference_signature(lib):
    """The library exports metal_ops::moe_block with the reference's mangled name."""
    out = subprocess.run(["nm", "-D", "--defined-only", lib.LIB_PATH], capture_output=True,
                         text=True).stdout
    ours = [l.split()[-1] for l in out.splitlines() if "metal_ops9moe_block" in l]
    assert len(ours) == 1
    ref_hdr = "/root/reference/src/gpu/metal_ops.hpp"
    if not os.path.exists(ref_hdr) or not shutil.which("g++"):
        pytest.skip("reference header not present")
    src = ('#include "%s"\nvoid f(){mvllm::metal_ops::moe_block(0,0,0,0,0,0,0,0,0,0,0,0,0,0,0,'
           '0,0,0);}\n' % ref_hdr)
    tmp = os.path.join(ROOT, "_work", "abi_probe")
    os.makedirs(tmp, exist_ok=True)
    with open(os.path.join(tmp, "p.cpp"), "w") as f:
        f.write(src)
    subprocess.run(["g++", "-std=c++17", "-c", os.path.join(tmp, "p.cpp"), "-o",
                    os.path.join(tmp, "p.o")], check=True)
    und = subprocess.run(["nm", "-u", os.path.join(tmp, "p.o")], capture_output=True,
                         text=True).stdout
    assert ours[0] in und


def test_invalid_arguments_rejected_without_gpu(lib):
    """metal_ops.cpp:452-457 argument checks return false before any device work."""
    c = cases.kat_identity(cases.ACT_SILU, 0.0)
    out = np.zeros((1, 4), np.float32)
    args = dict(g=c["g"], u=c["u"], d=c["d"], gs=None, us=None, ds=None, xg=c["xg"],
                xoff=c["xoff"], nr=c["nr"], rows=c["rows"], rw=c["rw"], out=out, S=1)
    assert lib.moe_block(0, 4, 4, 0, **args) is False
    assert lib.moe_block(1, 0, 4, 0, **args) is False
    assert lib.moe_block(1, 4, 4, 3, **args) is False
    bad = dict(args, xoff=None)
    assert lib.moe_block(1, 4, 4, 0, **bad) is False
    bad = dict(args, xg=None)
    assert lib.moe_block(1, 4, 4, 0, **bad) is False


def test_backend_identity_and_uninitialised_errors(lib):
    assert lib.backend_name() == "cuda-sm100a"
    if lib.available():
        pytest.skip("library already initialised in this process")
    c = cases.kat_identity(cases.ACT_SILU, 0.0)
    out = np.zeros((1, 4), np.float32)
    with pytest.raises(lib.MoeError) as ei:
        lib.moe_block(1, 4, 4, 0, c["g"], c["u"], c["d"], None, None, None, c["xg"], c["xoff"],
                      c["nr"], c["rows"], c["rw"], out, 1)
    assert ei.value.code == lib.ERR_NOT_INIT
    assert lib.lib().mvllm_moe_block_dev_workspace(0, 4, 4, 0, 1, 1, 1) == 0
    assert lib.lib().mvllm_moe_layer_workspace(4, 2, 8, 0, 512, 512, 7) > 0


def test_peer_window_layout_and_argument_checks(lib):
    """The exchange window's layout (a host function) and the peer entries'
    argument checks, which return before any device work."""
    D, K, N, seg = 7168, 8, 8, 1024
    total, off = lib.ep_window_layout(N, seg, K, D, lib.DTYPE_BF16)
    rows = N * seg
    assert off["x"] == 0
    assert off["ids"] >= rows * D * 2 and off["wt"] >= off["ids"] + rows * K * 4
    assert off["back"] >= off["wt"] + rows * K * 4
    assert total >= off["back"] + rows * lib.partial_row_bytes(D)
    assert all(v % 256 == 0 for v in off.values()) and total % 256 == 0
    assert total - off["back"] < rows * lib.partial_row_bytes(D) + 256
    f32, _ = lib.ep_window_layout(N, seg, K, D, lib.DTYPE_F32)
    assert f32 > total
    L = lib.lib()
    for bad in ((0, seg, K, D, 1), (33, seg, K, D, 1), (N, 0, K, D, 1), (N, seg, 17, D, 1),
                (N, seg, K, 12, 1), (N, seg, K, D, 5)):
        assert L.mvllm_moe_ep_window_layout(*bad, None) == 0
    with pytest.raises(lib.MoeError):
        lib.ep_window_layout(0, seg, K, D, lib.DTYPE_BF16)
    nul = C.c_void_p()
    assert L.mvllm_moe_peer_open(None, C.byref(nul)) == lib.ERR_INVALID
    assert L.mvllm_moe_peer_close(None) == lib.ERR_INVALID
    assert L.mvllm_moe_peer_free(None) == lib.ERR_INVALID
    assert L.mvllm_moe_peer_alloc(0, C.byref(nul), None) == lib.ERR_INVALID
    with pytest.raises(ValueError):
        lib.peer_open(b"short")
    p = C.c_void_p(4096)
    # dispatch: T above the segment, then nranks 0
    assert L.mvllm_moe_ep_dispatch_peer_dev(None, p, 1, p, p, 9, K, D, 384, N, None, None, 0, 8,
                                            p, p, p) == lib.ERR_INVALID
    assert L.mvllm_moe_ep_dispatch_peer_dev(None, p, 1, p, p, 8, K, D, 384, 0, None, None, 0, 8,
                                            p, p, p) == lib.ERR_INVALID
    # partial-peer: a window address that is not 256-byte aligned
    tabs = [p] * 6
    assert L.mvllm_moe_layer_partial_peer_dev(None, N, seg, 0, K, 48, D, 2048, 7, 1,
                                              C.c_void_p(4096 + 16), p, *tabs, 2, 4.0, 25.0,
                                              p, 1 << 30) == lib.ERR_INVALID


def test_init_without_gpu_reports_error(lib):
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("a GPU is present")
    except ImportError:
        pass
    rc = lib.lib().mvllm_moe_init(0)
    assert rc in (lib.ERR_CUDA, lib.ERR_INVALID)
    assert lib.last_error()


def _cpp_caller(lib):
    """Builds and runs tests/cpp_caller.cpp; returns its stdout."""
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    out_dir = os.path.join(root, "tests", "_build")
    os.makedirs(out_dir, exist_ok=True)
    exe = os.path.join(out_dir, "cpp_caller")
    libdir = os.path.dirname(lib.LIB_PATH)
    subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", "-Werror",
                    os.path.join(root, "tests", "cpp_caller.cpp"),
                    "-I" + os.path.join(root, "include"), "-L" + libdir, "-lmvllm_moe",
                    "-Wl,-rpath," + libdir, "-o", exe], check=True)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "CPP-CALLER-OK" in r.stdout
    return r.stdout


def test_cpp_caller_links_and_runs(lib):
    """A reference-style C++ translation unit links against the library through
    include/mvllm_metal_ops.hpp and runs (tests/cpp_caller.cpp): argument
    rejection and backend identity; the device call where a GPU is present."""
    _cpp_caller(lib)


@pytest.mark.gpu
def test_cpp_caller_device_call(lib):
    """The same C++ caller on a GPU: metal_ops::init and one moe_block call."""
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    assert "(no device)" not in _cpp_caller(lib)
