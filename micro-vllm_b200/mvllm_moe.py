"""Python host binding of libmvllm_moe.so (the sm_100a MoE block).

Mirrors the reference's operator interface for this path: ``moe_block`` has
the argument list, meaning and error behaviour of
``mvllm::metal_ops::moe_block`` (src/gpu/metal_ops.hpp:104-108): it returns
True on success and False exactly where the reference returns false; a CUDA
failure raises ``MoeError``.  There is no CPU fallback: importing this module
on a machine without the built library raises, and every call runs the CUDA
library.

Host buffers are numpy arrays; device buffers are torch CUDA tensors (torch is
only used for device memory and streams).
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libmvllm_moe.so")

OK, ERR_INVALID, ERR_CUDA, ERR_NOMEM, ERR_UNSUPPORTED, ERR_TIMEOUT, ERR_NOT_INIT, ERR_DEVICE, \
    ERR_WORKSPACE, ERR_RANGE, ERR_ACT_RANGE = range(11)
ACT_SILU, ACT_CLAMP_SWIGLU, ACT_SITU = 0, 1, 2
FMT_F32, FMT_INT4_G64, FMT_MXFP4, FMT_INT8_ROW, FMT_FP8_B128 = 0, 4, 7, 8, 9
DTYPE_F32, DTYPE_BF16 = 0, 1
SCORE_SIGMOID, SCORE_SQRT_SOFTPLUS = 0, 1
# Tensor-core (prefill) modes for MXFP4 experts (mvllm_moe.h MVLLM_PREFILL_*).
PREFILL_F16, PREFILL_MXF4_X1, PREFILL_MXF4_X2, PREFILL_MXF4_X3, PREFILL_MXF8_X1, \
    PREFILL_MXF8_X2 = range(6)
PREFILL_NAMES = ("f16", "mxf4x1", "mxf4x2", "mxf4x3", "mxf8x1", "mxf8x2")

# Every symbol include/mvllm_moe.h declares (checked by tests/test_abi.py).
C_SYMBOLS = (
    "mvllm_moe_init", "mvllm_moe_shutdown", "mvllm_moe_available", "mvllm_moe_backend_name",
    "mvllm_moe_last_error", "mvllm_moe_stats", "mvllm_moe_block", "mvllm_moe_cache_register",
    "mvllm_moe_cache_unregister", "mvllm_moe_cache_clear", "mvllm_moe_cache_bytes",
    "mvllm_moe_block_dev_workspace", "mvllm_moe_block_dev", "mvllm_moe_permute_workspace",
    "mvllm_moe_permute_dev", "mvllm_moe_layer_workspace", "mvllm_moe_layer_dev",
    "mvllm_moe_layer_host", "mvllm_quantize_int4_g64_dev", "mvllm_pack_mxfp4_dev",
    "mvllm_matmul_dev", "mvllm_moe_profile_enable", "mvllm_moe_profile_read",
    "mvllm_moe_permute_dev_noalloc", "mvllm_moe_ep_plan_dev", "mvllm_moe_ep_pack_dev",
    "mvllm_moe_ep_combine_dev", "mvllm_moe_topk_dev", "mvllm_moe_route_dev",
    "mvllm_moe_ep_combine16_dev", "mvllm_moe_layer_partial_dev", "mvllm_moe_tier_configure",
    "mvllm_moe_expert_bind", "mvllm_moe_expert_unbind", "mvllm_moe_tier_stats",
    "mvllm_moe_epilogue_workspace", "mvllm_moe_epilogue_dev", "mvllm_moe_host_register",
    "mvllm_moe_host_unregister", "mvllm_moe_route_ex_dev", "mvllm_moe_ep_local_ids_dev",
    "mvllm_moe_dense_ffn_workspace", "mvllm_moe_dense_ffn_dev", "mvllm_moe_wait_selftest",
    "mvllm_moe_set_prefill_mode", "mvllm_moe_get_prefill_mode", "mvllm_mx_terms_dev",
    "mvllm_moe_mma_rate", "mvllm_moe_set_sm_limit", "mvllm_moe_ep_plan_fixed_dev",
    "mvllm_moe_set_exact", "mvllm_moe_get_exact", "mvllm_moe_layer_error",
    "mvllm_moe_peer_alloc", "mvllm_moe_peer_open", "mvllm_moe_peer_close", "mvllm_moe_peer_free",
    "mvllm_moe_ep_window_layout", "mvllm_moe_ep_dispatch_peer_dev",
    "mvllm_moe_layer_partial_peer_dev",
)
PHASES = ("permute", "gather", "plan", "expert_phase1", "expert_phase2", "combine")


class MoeError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"mvllm_moe error {code}: {msg}")
        self.code = code


_lib = None


def lib():
    """Loads the CUDA library (fails loudly if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: run micro-vllm_b200/build.py")
        L = C.CDLL(LIB_PATH)
        vp, i, f, sz = C.c_void_p, C.c_int, C.c_float, C.c_size_t
        sig = {
            "mvllm_moe_init": (i, [i]),
            "mvllm_moe_shutdown": (None, []),
            "mvllm_moe_available": (i, []),
            "mvllm_moe_backend_name": (C.c_char_p, []),
            "mvllm_moe_last_error": (C.c_char_p, []),
            "mvllm_moe_stats": (None, [vp] * 6),
            "mvllm_moe_block": (i, [i, i, i, i, i] + [vp] * 6 + [vp] * 6 + [i, i, f, f]),
            "mvllm_moe_cache_register": (i, [vp, sz, C.c_uint64]),
            "mvllm_moe_cache_unregister": (i, [vp]),
            "mvllm_moe_cache_clear": (None, []),
            "mvllm_moe_cache_bytes": (sz, []),
            "mvllm_moe_block_dev_workspace": (sz, [i] * 7),
            "mvllm_moe_block_dev": (i, [vp, i, i, i, i] + [vp] * 6 + [vp, i, i] + [vp] * 5 +
                                    [i, i, f, f, i, vp, sz]),
            "mvllm_moe_permute_workspace": (sz, [i] * 4),
            "mvllm_moe_permute_dev": (i, [vp, vp, vp, i, i, i, i] + [vp] * 6 + [vp, sz]),
            "mvllm_moe_layer_workspace": (sz, [i] * 7),
            "mvllm_moe_layer_dev": (i, [vp] + [i] * 7 + [vp, vp, vp, i] + [vp] * 6 +
                                    [vp, i, f, f, vp, sz]),
            "mvllm_moe_layer_host": (i, [i] * 7 + [vp] * 3 + [vp] * 6 + [vp, i, f, f]),
            "mvllm_quantize_int4_g64_dev": (i, [vp, vp, i, i, vp, vp]),
            "mvllm_pack_mxfp4_dev": (i, [vp, vp, i, i, vp, vp]),
            "mvllm_matmul_dev": (i, [vp, i, vp, vp, vp, vp, i, i, i]),
            "mvllm_moe_profile_enable": (None, [i]),
            "mvllm_moe_profile_read": (i, [vp, vp, i]),
            "mvllm_moe_permute_dev_noalloc": (i, [vp, vp, vp, i, i, i, i] + [vp] * 6),
            "mvllm_moe_ep_plan_dev": (i, [vp, vp, i, i, i, i, vp, i, vp, vp]),
            "mvllm_moe_ep_pack_dev": (i, [vp, vp, i, vp, vp, i, i, i, i, i, vp, vp, i, vp, vp, vp,
                                          vp]),
            "mvllm_moe_ep_combine_dev": (i, [vp, vp, vp, i, i, i, vp]),
            "mvllm_moe_ep_combine16_dev": (i, [vp, vp, vp, i, i, i, vp]),
            "mvllm_moe_tier_configure": (i, [sz, sz]),
            "mvllm_moe_host_register": (i, [vp, sz]),
            "mvllm_moe_host_unregister": (i, [vp]),
            "mvllm_moe_epilogue_workspace": (sz, [i, i, i]),
            "mvllm_moe_epilogue_dev": (i, [vp, i, i, i, vp, vp, f, i, vp, vp, f, vp, vp, vp, sz]),
            "mvllm_moe_expert_bind": (i, [vp, sz, C.c_uint64]),
            "mvllm_moe_expert_unbind": (i, [vp]),
            "mvllm_moe_tier_stats": (None, [vp] * 7),
            "mvllm_moe_layer_partial_dev": (i, [vp] + [i] * 7 + [vp, vp, vp, i] + [vp] * 6 +
                                            [vp, i, f, f, vp, sz]),
            "mvllm_moe_topk_dev": (i, [vp, vp, vp, i, i, i, vp, vp]),
            "mvllm_moe_route_dev": (i, [vp, vp, i, i, i, vp, vp, i, i, vp, vp, vp, vp]),
            "mvllm_moe_route_ex_dev": (i, [vp, vp, i, i, i, vp, vp, i, i, i, f, vp, vp, vp, vp]),
            "mvllm_moe_ep_local_ids_dev": (i, [vp, vp, i, i, i, i, vp, vp, i, vp]),
            "mvllm_moe_dense_ffn_workspace": (sz, [i, i, i]),
            "mvllm_moe_wait_selftest": (i, [vp, vp]),
            "mvllm_moe_set_prefill_mode": (i, [i]),
            "mvllm_moe_get_prefill_mode": (i, []),
            "mvllm_moe_set_exact": (i, [i]),
            "mvllm_moe_layer_error": (i, [vp, vp]),
            "mvllm_moe_get_exact": (i, []),
            "mvllm_mx_terms_dev": (i, [vp, i, vp, i, i, vp, vp]),
            "mvllm_moe_mma_rate": (i, [i, i, i, i, vp]),
            "mvllm_moe_set_sm_limit": (i, [i]),
            "mvllm_moe_ep_plan_fixed_dev": (i, [vp, vp, i, i, i, i, vp, i, i, vp, vp]),
            "mvllm_moe_peer_alloc": (i, [sz, vp, vp]),
            "mvllm_moe_peer_open": (i, [vp, vp]),
            "mvllm_moe_peer_close": (i, [vp]),
            "mvllm_moe_peer_free": (i, [vp]),
            "mvllm_moe_ep_window_layout": (sz, [i, i, i, i, i, vp]),
            "mvllm_moe_ep_dispatch_peer_dev": (i, [vp, vp, i, vp, vp] + [i] * 5 +
                                               [vp, vp, i, i, vp, vp, vp]),
            "mvllm_moe_layer_partial_peer_dev": (i, [vp] + [i] * 9 + [vp, vp] + [vp] * 6 +
                                                 [i, f, f, vp, sz]),
            "mvllm_moe_dense_ffn_dev": (i, [vp, i, i, i, i] + [vp] * 7 + [i, f, f, vp, i, vp,
                                                                         sz]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    return lib().mvllm_moe_last_error().decode()


def _check(rc):
    if rc != OK:
        raise MoeError(rc, last_error())


def init(device: int = 0) -> None:
    _check(lib().mvllm_moe_init(device))


def shutdown() -> None:
    lib().mvllm_moe_shutdown()


def set_prefill_mode(mode) -> None:
    """Tensor-core mode for MXFP4 experts: a PREFILL_* value or its name;
    -1 (or None) restores the default."""
    if mode is None:
        mode = -1
    if isinstance(mode, str):
        mode = PREFILL_NAMES.index(mode)
    _check(lib().mvllm_moe_set_prefill_mode(int(mode)))


def get_prefill_mode() -> int:
    return int(lib().mvllm_moe_get_prefill_mode())


def set_exact(on) -> None:
    """Exact mode for the layer epilogue and the router scores: True keeps the
    reference's summation order (bit-identical), False the tolerance-mode
    kernels, None the default (MVLLM_EXACT, else off)."""
    _check(lib().mvllm_moe_set_exact(-1 if on is None else int(bool(on))))


def get_exact() -> bool:
    return bool(lib().mvllm_moe_get_exact())


def set_sm_limit(sms: int) -> None:
    """SMs the persistent expert kernels fill (0: all)."""
    _check(lib().mvllm_moe_set_sm_limit(int(sms)))


def mma_rate(kind, n, pair, iters=20000) -> float:
    """Dense TFLOP/s of back-to-back MMAs (kind 0 mxf4, 1 mxf8f6f4, 2 f16)."""
    v = C.c_double(0.0)
    _check(lib().mvllm_moe_mma_rate(int(kind), int(n), int(pair), int(iters), C.byref(v)))
    return v.value


def mx_terms_dev(mode, src, planes, codes, stream=None) -> None:
    """Block-scaled terms of f16 device rows src [rows, K] (mvllm_mx_terms_dev)."""
    if isinstance(mode, str):
        mode = PREFILL_NAMES.index(mode)
    rows, K = src.shape
    _check(lib().mvllm_mx_terms_dev(_stream(stream), int(mode), C.c_void_p(src.data_ptr()),
                                    rows, K, C.c_void_p(planes.data_ptr()),
                                    C.c_void_p(codes.data_ptr())))


def available() -> bool:
    return bool(lib().mvllm_moe_available())


def backend_name() -> str:
    return lib().mvllm_moe_backend_name().decode()


def stats():
    vals = [C.c_uint64(), C.c_uint64(), C.c_uint64(), C.c_double(), C.c_double(), C.c_double()]
    lib().mvllm_moe_stats(*[C.byref(v) for v in vals])
    return {"calls": vals[0].value, "experts": vals[1].value, "rows": vals[2].value,
            "h2d_ms": vals[3].value, "kernel_ms": vals[4].value, "d2h_ms": vals[5].value}


def profile_enable(on: bool = True) -> None:
    lib().mvllm_moe_profile_enable(1 if on else 0)


def profile_read():
    """{phase: (device ms, launches)} since profile_enable."""
    n = len(PHASES)
    ms = (C.c_double * n)()
    cnt = (C.c_longlong * n)()
    lib().mvllm_moe_profile_read(ms, cnt, n)
    return {PHASES[i]: (ms[i], cnt[i]) for i in range(n)}


def _p(a):
    return None if a is None else C.c_void_p(a.ctypes.data)


def _parr(arrs):
    """Pointer array for the C ABI: a list of numpy arrays (their data
    pointers), or a contiguous int64 numpy array of addresses passed in place."""
    if arrs is None:
        return None
    if isinstance(arrs, np.ndarray) and arrs.dtype in (np.int64, np.uint64) and arrs.ndim == 1:
        return C.cast(arrs.ctypes.data, C.POINTER(C.c_void_p))
    out = (C.c_void_p * len(arrs))()
    for k, a in enumerate(arrs):
        out[k] = None if a is None else a.ctypes.data
    return out


# --------------------------------------------------------------- host path --
def moe_block(nb, D, Iinter, fmt, g, u, d, gs, us, ds, xg, xoff, nr, rows, rw, out, S, act=0,
              act_a=0.0, act_b=0.0, qgs=0) -> bool:
    """metal_ops::moe_block on host numpy buffers (``out`` is accumulated in place).

    Returns False where the reference returns false (invalid arguments);
    raises MoeError on a CUDA failure.
    """
    rc = lib().mvllm_moe_block(nb, D, Iinter, fmt, qgs, _parr(g), _parr(u), _parr(d), _parr(gs),
                               _parr(us), _parr(ds), _p(xg), _p(xoff), _p(nr), _p(rows), _p(rw),
                               _p(out), S, act, act_a, act_b)
    if rc == ERR_INVALID:
        return False
    _check(rc)
    return True


def host_register(arr: np.ndarray) -> None:
    """Page-locks a host array for the host-pointer entries (see the header)."""
    _check(lib().mvllm_moe_host_register(arr.ctypes.data, arr.nbytes))


def host_unregister(arr: np.ndarray) -> None:
    _check(lib().mvllm_moe_host_unregister(arr.ctypes.data))


def tier_configure(budget_bytes: int, slot_bytes: int) -> None:
    _check(lib().mvllm_moe_tier_configure(budget_bytes, slot_bytes))


def expert_bind(arr: np.ndarray, generation: int = 0) -> None:
    """Binds a host blob (a numpy array, e.g. one expert's packed arrays in
    one buffer) to the device expert tier."""
    _check(lib().mvllm_moe_expert_bind(arr.ctypes.data, arr.nbytes, generation))


def expert_unbind(arr: np.ndarray) -> None:
    _check(lib().mvllm_moe_expert_unbind(arr.ctypes.data))


def tier_stats():
    v = [C.c_uint64() for _ in range(6)] + [C.c_size_t()]
    lib().mvllm_moe_tier_stats(*[C.byref(x) for x in v])
    keys = ("hits", "misses", "evictions", "bytes_in", "overflow", "overflow_bytes",
            "resident_bytes")
    return {k: x.value for k, x in zip(keys, v)}


def cache_register(arr: np.ndarray, generation: int = 0) -> None:
    _check(lib().mvllm_moe_cache_register(C.c_void_p(arr.ctypes.data), arr.nbytes, generation))


def cache_unregister(arr: np.ndarray) -> None:
    _check(lib().mvllm_moe_cache_unregister(C.c_void_p(arr.ctypes.data)))


def cache_clear() -> None:
    lib().mvllm_moe_cache_clear()


def cache_bytes() -> int:
    return lib().mvllm_moe_cache_bytes()


def _addr_array(t):
    """A table of device addresses for the C ABI: a contiguous int64/uint64
    numpy array is passed in place, any other sequence of ints is copied."""
    if isinstance(t, np.ndarray) and t.dtype in (np.int64, np.uint64) and t.ndim == 1 \
            and t.flags["C_CONTIGUOUS"]:
        return C.cast(t.ctypes.data, C.POINTER(C.c_void_p))
    return (C.c_void_p * len(t))(*t)


def layer_host(T, K, E, n_shared, D, Iinter, fmt, idx, wt, x, tables, out, act, act_a=0.0,
               act_b=0.0):
    """Routed layer with host activations/routing and device-resident weights.

    ``tables`` holds six sequences of device addresses (ints, or int64 numpy
    arrays, which are passed without a copy): g, u, d, gs, us, ds.
    """
    arrs = [_addr_array(t) for t in tables]
    _check(lib().mvllm_moe_layer_host(T, K, E, n_shared, D, Iinter, fmt, _p(idx), _p(wt), _p(x),
                                      *arrs, _p(out), act, act_a, act_b))


# -------------------------------------------------------------- device path --
def _dp(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _stream(stream):
    if stream is None:
        import torch
        stream = torch.cuda.current_stream()
    return C.c_void_p(stream.cuda_stream)


def layer_workspace_bytes(T, K, E, n_shared, D, Iinter, fmt) -> int:
    return lib().mvllm_moe_layer_workspace(T, K, E, n_shared, D, Iinter, fmt)


def layer_dev(T, K, E, n_shared, D, Iinter, fmt, idx, wt, x, tables, out, act, act_a, act_b,
              workspace, stream=None):
    """Routed layer on device tensors; ``tables`` = six int64 CUDA tensors of addresses."""
    x_dtype = DTYPE_BF16 if str(x.dtype) == "torch.bfloat16" else DTYPE_F32
    _check(lib().mvllm_moe_layer_dev(_stream(stream), T, K, E, n_shared, D, Iinter, fmt, _dp(idx),
                                     _dp(wt), _dp(x), x_dtype, *[_dp(t) for t in tables],
                                     _dp(out), act, act_a, act_b, _dp(workspace),
                                     workspace.numel() * workspace.element_size()))


def layer_error(workspace, stream=None) -> int:
    """The device-side status of the last layer_dev / layer_partial_dev call
    that used ``workspace`` (synchronises the stream): 0 or an ERR_* code."""
    rc = int(lib().mvllm_moe_layer_error(_stream(stream), _dp(workspace)))
    if rc in (ERR_INVALID, ERR_CUDA):
        _check(rc)
    return rc


def partial_row_bytes(D) -> int:
    """Pitch of a partial row (mvllm_moe_layer_partial_dev): D f16 + 16-byte tail."""
    return 2 * D + 16


def layer_partial_dev(T, K, E, n_shared, D, Iinter, fmt, idx, wt, x, tables, out16, act, act_a,
                      act_b, workspace, stream=None):
    """The routed layer into partial rows: ``out16`` is a uint8 CUDA tensor of
    [T, partial_row_bytes(D)] (see decode_partial_rows)."""
    x_dtype = DTYPE_BF16 if str(x.dtype) == "torch.bfloat16" else DTYPE_F32
    _check(lib().mvllm_moe_layer_partial_dev(
        _stream(stream), T, K, E, n_shared, D, Iinter, fmt, _dp(idx), _dp(wt), _dp(x), x_dtype,
        *[_dp(t) for t in tables], _dp(out16), act, act_a, act_b, _dp(workspace),
        workspace.numel() * workspace.element_size()))


def decode_partial_rows(torch, rows, D):
    """f32 values of partial rows (uint8 [R, 2*D + 16]) -- for checks and tests."""
    h = rows[:, :2 * D].contiguous().view(torch.float16).float()
    sc = rows[:, 2 * D:2 * D + 4].contiguous().view(torch.float32)
    return h * sc


def block_dev_workspace_bytes(nb, D, Iinter, fmt, rows_cap, x_rows, S) -> int:
    return lib().mvllm_moe_block_dev_workspace(nb, D, Iinter, fmt, rows_cap, x_rows, S)


def block_dev(nb, D, Iinter, fmt, tables, x, x_rows, xoff, nr, rows, rw, out, S, act, act_a,
              act_b, rows_cap, workspace, stream=None):
    x_dtype = DTYPE_BF16 if str(x.dtype) == "torch.bfloat16" else DTYPE_F32
    _check(lib().mvllm_moe_block_dev(_stream(stream), nb, D, Iinter, fmt,
                                     *[_dp(t) for t in tables], _dp(x), x_dtype, x_rows,
                                     _dp(xoff), _dp(nr), _dp(rows), _dp(rw), _dp(out), S, act,
                                     act_a, act_b, rows_cap, _dp(workspace),
                                     workspace.numel() * workspace.element_size()))


def permute_workspace_bytes(T, K, E, n_shared) -> int:
    return lib().mvllm_moe_permute_workspace(T, K, E, n_shared)


def permute_dev(idx, wt, E, n_shared, nr, xoff, rows, rw, tok_pos, n_rows, workspace,
                stream=None):
    T, K = idx.shape
    _check(lib().mvllm_moe_permute_dev(_stream(stream), _dp(idx), _dp(wt), T, K, E, n_shared,
                                       _dp(nr), _dp(xoff), _dp(rows), _dp(rw), _dp(tok_pos),
                                       _dp(n_rows), _dp(workspace),
                                       workspace.numel() * workspace.element_size()))


def quantize_int4_g64_dev(w, packed, scales, stream=None):
    O, I = w.shape
    _check(lib().mvllm_quantize_int4_g64_dev(_stream(stream), _dp(w), O, I, _dp(packed),
                                             _dp(scales)))


def pack_mxfp4_dev(w, packed, scales, stream=None):
    O, I = w.shape
    _check(lib().mvllm_pack_mxfp4_dev(_stream(stream), _dp(w), O, I, _dp(packed), _dp(scales)))


def matmul_dev(fmt, y, x, w, scales, stream=None):
    S, I = x.shape
    O = y.shape[1]
    _check(lib().mvllm_matmul_dev(_stream(stream), fmt, _dp(y), _dp(x), _dp(w), _dp(scales), S,
                                  I, O))


# ----------------------------------------------------------- layer epilogue --
def epilogue_dev(acc, h, routed_scale=1.0, lat_n=None, eps=1e-6, up_fmt=0, up_w=None,
                 up_scales=None, shared=None, workspace=None, stream=None):
    """h += (lat_up . rmsnorm(acc)) * routed_scale + shared (device tensors)."""
    T, L = acc.shape
    H = h.shape[1]
    ws = workspace
    _check(lib().mvllm_moe_epilogue_dev(
        _stream(stream), T, H, L, _dp(acc), _dp(lat_n), eps, up_fmt, _dp(up_w), _dp(up_scales),
        routed_scale, _dp(shared), _dp(h), _dp(ws),
        0 if ws is None else ws.numel() * ws.element_size()))


def epilogue_workspace_bytes(T, H, L) -> int:
    return lib().mvllm_moe_epilogue_workspace(T, H, L)


# -------------------------------------------------------- expert parallelism --
def ep_plan_dev(idx, E, nranks, pos, send_cnt, dest=None, self_rank=0, stream=None):
    """pos [T, nranks] int32, send_cnt [nranks] int32 (device).  dest: device
    int32 [E] placement (rank, or -1 = replicated), None = strided."""
    T, K = idx.shape
    _check(lib().mvllm_moe_ep_plan_dev(_stream(stream), _dp(idx), T, K, E, nranks, _dp(dest),
                                       self_rank, _dp(pos), _dp(send_cnt)))


def ep_plan_fixed_dev(idx, E, nranks, capacity, pos, send_cnt, dest=None, self_rank=0,
                      stream=None):
    """The plan with destination d's rows at d * capacity (no host counts)."""
    T, K = idx.shape
    _check(lib().mvllm_moe_ep_plan_fixed_dev(_stream(stream), _dp(idx), T, K, E, nranks,
                                             _dp(dest), self_rank, capacity, _dp(pos),
                                             _dp(send_cnt)))


def ep_pack_dev(x, idx, wt, E, nranks, pos, send_x, send_idx, send_wt, dest=None, lid=None,
                self_rank=0, stream=None):
    T, K = idx.shape
    D = x.shape[1]
    x_dtype = DTYPE_BF16 if str(x.dtype) == "torch.bfloat16" else DTYPE_F32
    _check(lib().mvllm_moe_ep_pack_dev(_stream(stream), _dp(x), x_dtype, _dp(idx), _dp(wt), T, K,
                                       D, E, nranks, _dp(dest), _dp(lid), self_rank, _dp(pos),
                                       _dp(send_x), _dp(send_idx), _dp(send_wt)))


# ---- the exchange over peer memory (windows mapped through CUDA IPC)
PEER_HANDLE_BYTES = 64


def _ptr(v):
    """A device pointer from a tensor or a raw integer address."""
    if v is None or isinstance(v, int):
        return C.c_void_p(v)
    return C.c_void_p(v.data_ptr())


def peer_alloc(nbytes):
    """A new zeroed device window: (address, 64-byte IPC handle)."""
    p = C.c_void_p()
    h = (C.c_ubyte * PEER_HANDLE_BYTES)()
    _check(lib().mvllm_moe_peer_alloc(nbytes, C.byref(p), h))
    return p.value, bytes(h)


def peer_open(handle: bytes) -> int:
    """Maps another process's window from its handle; returns the address."""
    if len(handle) != PEER_HANDLE_BYTES:
        raise ValueError("an IPC handle has 64 bytes")
    p = C.c_void_p()
    h = (C.c_ubyte * PEER_HANDLE_BYTES).from_buffer_copy(handle)
    _check(lib().mvllm_moe_peer_open(h, C.byref(p)))
    return p.value


def peer_close(addr: int) -> None:
    _check(lib().mvllm_moe_peer_close(C.c_void_p(addr)))


def peer_free(addr: int) -> None:
    _check(lib().mvllm_moe_peer_free(C.c_void_p(addr)))


def ep_window_layout(nranks, seg, K, D, x_dtype):
    """(window bytes, {"x", "ids", "wt", "back"} byte offsets)."""
    off = (C.c_size_t * 4)()
    total = lib().mvllm_moe_ep_window_layout(nranks, seg, K, D, x_dtype, off)
    if total == 0:
        raise MoeError(ERR_INVALID, "ep_window_layout: invalid arguments")
    return total, dict(zip(("x", "ids", "wt", "back"), list(off)))


def ep_dispatch_peer_dev(x, idx, wt, E, nranks, seg, pos, send_cnt, windows, dest=None, lid=None,
                         self_rank=0, stream=None):
    """Token rows, local ids and weights stored into the ranks' windows
    (windows: device int64 [nranks] of window addresses)."""
    T, K = idx.shape
    D = x.shape[1]
    x_dtype = DTYPE_BF16 if str(x.dtype) == "torch.bfloat16" else DTYPE_F32
    _check(lib().mvllm_moe_ep_dispatch_peer_dev(
        _stream(stream), _dp(x), x_dtype, _dp(idx), _dp(wt), T, K, D, E, nranks, _dp(dest),
        _dp(lid), self_rank, seg, _dp(pos), _dp(send_cnt), _dp(windows)))


def layer_partial_peer_dev(nranks, seg, self_rank, K, E, D, Iinter, fmt, x_dtype, window,
                           windows, tables, act, act_a, act_b, workspace, stream=None):
    """The rank's experts over its own window's rows, partial rows stored into
    the owners' windows (window: own address; windows: device int64 [nranks])."""
    _check(lib().mvllm_moe_layer_partial_peer_dev(
        _stream(stream), nranks, seg, self_rank, K, E, D, Iinter, fmt, x_dtype,
        C.c_void_p(window), _dp(windows), *[_dp(t) for t in tables], act, act_a, act_b,
        _dp(workspace), workspace.numel() * workspace.element_size()))


def ep_combine_dev(back, pos, out, stream=None):
    T, nranks = pos.shape
    D = out.shape[1]
    _check(lib().mvllm_moe_ep_combine_dev(_stream(stream), _dp(back), _dp(pos), T, nranks, D,
                                          _dp(out)))


def ep_combine16_dev(back16, pos, out, stream=None):
    """back16: a uint8 tensor of partial rows or the raw address of a
    window's back region."""
    T, nranks = pos.shape
    D = out.shape[1]
    _check(lib().mvllm_moe_ep_combine16_dev(_stream(stream), _ptr(back16), _dp(pos), T, nranks,
                                            D, _dp(out)))


# ------------------------------------------------------------------ routing --
def topk_dev(choice, K, idx, wt, mix=None, stream=None):
    """Device moe_topk over the rows of choice [T, E]."""
    T, E = choice.shape
    _check(lib().mvllm_moe_topk_dev(_stream(stream), _dp(choice), _dp(mix), T, E, K, _dp(idx),
                                    _dp(wt)))


def route_ex_dev(x, router, bias, K, idx, wt, scores, choice, score_fn=SCORE_SIGMOID,
                 routed_scale=1.0, stream=None):
    """Router scores (score_fn of x . router^T, + bias), top-K and the weights
    times routed_scale, on device.  SCORE_SQRT_SOFTPLUS with K=6 is
    DeepSeek-V4's route (dsv4_cuda.cpp:1541-1587)."""
    T, H = x.shape
    E = router.shape[0]
    x_dtype = DTYPE_BF16 if str(x.dtype) == "torch.bfloat16" else DTYPE_F32
    _check(lib().mvllm_moe_route_ex_dev(_stream(stream), _dp(x), x_dtype, T, H, _dp(router),
                                        _dp(bias), E, K, score_fn, routed_scale, _dp(idx),
                                        _dp(wt), _dp(scores), _dp(choice)))


def ep_local_ids_dev(idx, E, nranks, self_rank, local_idx, dest=None, lid=None, stream=None):
    """local_idx [T, K] = the local id of each slot rank self_rank serves, else -1."""
    T, K = idx.shape
    _check(lib().mvllm_moe_ep_local_ids_dev(_stream(stream), _dp(idx), T, K, E, nranks, _dp(dest),
                                            _dp(lid), self_rank, _dp(local_idx)))


def wait_selftest():
    """(completed, timed_out) of the bounded-wait health check (about 2 s)."""
    a, b = C.c_int(0), C.c_int(0)
    _check(lib().mvllm_moe_wait_selftest(C.byref(a), C.byref(b)))
    return bool(a.value), bool(b.value)


def dense_ffn_workspace_bytes(T, H, O) -> int:
    return lib().mvllm_moe_dense_ffn_workspace(T, H, O)


def dense_ffn_dev(fmt, x, gate, up, down, y, act, act_a=0.0, act_b=0.0, accumulate=False,
                  workspace=None, stream=None):
    """y (+)= down . act(gate . x, up . x) on device; gate/up/down = (weights,
    scales-or-None) device tensors in format fmt; x [T, H], y [T, H] f32."""
    import torch
    T, H = x.shape
    O = gate[0].shape[0]
    ws = workspace
    if ws is None:
        ws = torch.empty(dense_ffn_workspace_bytes(T, H, O), dtype=torch.uint8, device=x.device)
    _check(lib().mvllm_moe_dense_ffn_dev(
        _stream(stream), fmt, T, H, O, _dp(gate[0]), _dp(gate[1]), _dp(up[0]), _dp(up[1]),
        _dp(down[0]), _dp(down[1]), _dp(x), act, act_a, act_b, _dp(y), 1 if accumulate else 0,
        _dp(ws), ws.numel() * ws.element_size()))


def route_dev(x, router, bias, K, idx, wt, scores, choice, stream=None):
    """Router scores (sigmoid of x . router^T, + bias) and top-K on device."""
    T, H = x.shape
    E = router.shape[0]
    x_dtype = DTYPE_BF16 if str(x.dtype) == "torch.bfloat16" else DTYPE_F32
    _check(lib().mvllm_moe_route_dev(_stream(stream), _dp(x), x_dtype, T, H, _dp(router),
                                     _dp(bias), E, K, _dp(idx), _dp(wt), _dp(scores),
                                     _dp(choice)))
