"""ctypes binding of libhelix_kv.so, the C ABI in include/helix_kv.h.

Torch is used here for device memory and streams only: every call passes raw
device pointers and the current CUDA stream to the library. There is no CPU
path; a missing library or a CPU tensor raises.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

_HERE = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("HELIX_KV_LIB", _HERE / "libhelix_kv.so"))

# status and device error bits (helix_kv.h)
HX_OK, HX_ERR_ARG, HX_ERR_UNSUPPORTED, HX_ERR_LAUNCH, HX_ERR_SCRATCH_LIMIT = 0, 1, 2, 3, 4
DEV_ERR = {0x1: "outlier arena full", 0x2: "index out of range", 0x4: "bounded wait ran out",
           0x8: "selection threshold not isolated"}
SEL_DENSE, SEL_THRESHOLD, SEL_LIST, SEL_SLICES = 0, 1, 2, 3
VPOS_PHYSICAL = 0x100  # OR-ed into the decode's sel_mode (helix_kv.h)
DECODE_CUDA_CORES = 0x200  # OR-ed into sel_mode: QK and PV in FFMA (helix_kv.h)

c_vp, c_i32, c_i64, c_f32 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_float


class LayerScales(ctypes.Structure):
    _fields_ = [("k_poles", c_vp), ("k_upper", c_vp), ("k_lower", c_vp),
                ("v_poles", c_vp), ("v_upper", c_vp), ("v_lower", c_vp),
                ("levels_k", c_i32), ("levels_v", c_i32), ("t_cal", c_i32), ("reserved", c_i32),
                ("k_thresh", c_vp), ("v_thresh", c_vp)]


class PoolLayer(ctypes.Structure):
    _fields_ = [("codes", c_vp), ("stats", c_vp), ("dir", c_vp), ("arena", c_vp), ("arena_top", c_vp),
                ("arena_capacity", c_i64), ("num_blocks", c_i32), ("block_size", c_i32),
                ("num_kv_heads", c_i32), ("head_size", c_i32), ("bits_k", c_i32), ("bits_v", c_i32)]


_P = ctypes.POINTER
_SIGS = {
    "hx_version": (ctypes.c_char_p, []),
    "hx_pool_init": (c_i32, [c_vp, _P(PoolLayer)]),
    "hx_pool_reset_pages": (c_i32, [c_vp, _P(PoolLayer), c_vp, c_i32, c_vp]),
    "hx_pack_append": (c_i32, [c_vp, _P(PoolLayer), _P(LayerScales), c_vp, c_vp, c_vp, c_vp, c_i32, c_vp]),
    "hx_scales_prepare": (c_i32, [c_vp, _P(LayerScales), c_i32, c_i32, c_vp, c_vp]),
    "hx_unpack_pages": (c_i32, [c_vp, _P(PoolLayer), _P(LayerScales), c_vp, c_vp, c_i32, c_vp, c_vp, c_vp]),
    "hx_nuq_pack_dense": (c_i32, [c_vp, c_i32, c_vp, c_vp, c_vp, c_vp, c_i32, c_i32, c_i32, c_i32,
                                  c_vp, c_vp, c_vp]),
    "hx_nuq_unpack_dense": (c_i32, [c_vp, c_i32, c_vp, c_vp, c_vp, c_vp, c_i32, c_i32, c_i32, c_i32, c_vp]),
    "hx_nuq_quantize_flat": (c_i32, [c_vp, c_i32, c_vp, c_vp, c_vp, c_vp, c_i64, c_i32, c_i32, c_i64,
                                     c_i64, c_i64, c_i32, c_vp, c_vp, c_vp]),
    "hx_nuq_dequantize_flat": (c_i32, [c_vp, c_i32, c_vp, c_vp, c_vp, c_vp, c_i64, c_i32, c_vp, c_vp]),
    "hx_page_stats": (c_i32, [c_vp, c_i32, c_vp, c_i32, c_i32, c_i32, c_i32, c_vp, c_vp]),
    "hx_quest_scores": (c_i32, [c_vp, c_vp, c_i32, c_i32, c_i32, c_i32, c_i32, c_i32, c_vp, c_vp, c_i64,
                                c_i64, c_vp, c_i32, c_vp, c_i32, c_i32, c_i32, c_vp, c_vp]),
    "hx_quest_threshold": (c_i32, [c_vp, c_vp, c_i32, c_i32, c_vp, c_i32, c_i32, c_i32, c_i32, c_i32,
                                   c_i32, c_i32, c_vp, c_vp, c_vp, c_vp, c_vp]),
    "hx_quest_slices": (c_i32, [c_i32]),
    "hx_quest_threshold_slices": (c_i32, [c_vp, c_vp, c_i32, c_i32, c_vp, c_i32, c_i32, c_i32, c_i32, c_i32,
                                          c_i32, c_i32, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp]),
    "hx_quest_compact": (c_i32, [c_vp, c_vp, c_vp, c_i32, c_i32, c_vp, c_i32, c_i32, c_i32, c_i32, c_i32,
                                 c_vp, c_vp]),
    "hx_quest_lists": (c_i32, [c_vp, c_vp, c_vp, c_i32, c_i32, c_vp, c_i32, c_i32, c_i32, c_i32, c_vp, c_vp, c_vp]),
    "hx_quest_localize": (c_i32, [c_vp, c_vp, c_vp, c_i32, c_i32, c_vp, c_i32, c_i32, c_i32, c_i32, c_vp, c_vp]),
    "hx_decode_scratch_bytes": (c_i64, [c_i32, c_i32, c_i32]),
    "hx_decode_attn": (c_i32, [c_vp, _P(PoolLayer), _P(LayerScales), c_vp, c_i32, c_i32, c_f32, c_vp, c_i32,
                               c_vp, c_i32, c_i32, c_i32, c_vp, c_vp, c_i32, c_vp, c_i32, c_vp, c_i32,
                               c_vp, c_vp, c_vp, c_vp, c_vp]),
    "hx_calib_scratch_bytes": (c_i64, [c_i32, c_i64]),
    "hx_calib_rows": (c_i32, [c_vp, c_vp, c_i32, c_i64, ctypes.c_double, ctypes.c_double, c_i32, c_i32, c_vp, c_vp,
                              c_vp, c_vp, c_vp]),
    "hx_decode_attn_select": (c_i32, [c_vp, _P(PoolLayer), _P(LayerScales), c_vp, c_i32, c_i32, c_f32, c_vp, c_i32,
                                      c_vp, c_i32, c_i32, c_i32, c_vp, c_vp, c_i32, c_i32, c_i32, c_i32, c_i32,
                                      c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp]),
    "hx_prefill_attn": (c_i32, [c_vp, _P(PoolLayer), _P(LayerScales), c_vp, c_vp, c_i32, c_i32, c_f32, c_vp, c_i32,
                                c_vp, c_i32, c_i32, c_vp, c_vp, c_vp, c_vp]),
    "hx_decode_attn_noalloc": (c_i32, [c_vp, _P(PoolLayer), _P(LayerScales), c_vp, c_i32, c_i32, c_f32, c_vp,
                                       c_i32, c_vp, c_i32, c_i32, c_i32, c_vp, c_vp, c_i32, c_vp, c_i32, c_vp,
                                       c_i32, c_vp, c_vp, c_vp, c_vp]),
    "hx_merge_partials": (c_i32, [c_vp, c_vp, c_vp, c_i32, c_i32, c_i32, c_vp, c_vp, c_vp]),
    "hx_merge_gathered": (c_i32, [c_vp, c_vp, c_i32, c_i32, c_i32, c_vp, c_vp, c_vp]),
    "hx_exchange_merge": (c_i32, [c_vp, c_vp, c_vp, c_i32, c_i32, c_i32, c_i32, c_i32, c_vp, c_vp, c_vp,
                                  ctypes.c_uint32, c_vp]),
    "hx_selected_attention": (c_i32, [c_vp, c_i32, c_vp, c_vp, c_vp, c_vp, c_i32, c_i32, c_i32, c_i32,
                                      c_i32, c_i32, c_f32, c_vp]),
}

_lib = None
_lock = threading.Lock()


class HelixError(RuntimeError):
    pass


def lib():
    """The loaded library; raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise HelixError(
                    f"{LIB_PATH} is missing: the helix KV path has no CPU fallback. Build it with "
                    "`python helix-lite_b200/hxlib/build.py` (or __graft_entry__.build()).")
            L = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in _SIGS.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


# kernel launches each entry point makes (bench.py counts launches with this)
LAUNCHES = {"hx_scales_prepare": 2, "hx_pool_init": 1, "hx_pool_reset_pages": 1, "hx_pack_append": lambda a: 2 if a[7] <= 32768 else 3, "hx_unpack_pages": 1,
            "hx_nuq_pack_dense": 1, "hx_nuq_unpack_dense": 1, "hx_nuq_quantize_flat": 2,
            "hx_nuq_dequantize_flat": 1, "hx_page_stats": 1, "hx_quest_scores": 1, "hx_quest_threshold": lambda a: 1 if a[11] else 2,
            "hx_quest_threshold_slices": lambda a: 1 if a[11] else 2, "hx_quest_localize": 1,
            "hx_quest_compact": 1, "hx_quest_lists": 2, "hx_decode_attn": 1, "hx_decode_attn_noalloc": 1, "hx_prefill_attn": 1, "hx_calib_rows": 1, "hx_decode_attn_select": 1, "hx_merge_partials": 1, "hx_merge_gathered": 1, "hx_exchange_merge": 1,
            "hx_selected_attention": 1}
launch_count = [0]


def call(name, *args):
    n = LAUNCHES.get(name, 0)
    launch_count[0] += n(args) if callable(n) else n
    rc = getattr(lib(), name)(*args)
    if rc != HX_OK:
        what = {HX_ERR_ARG: "invalid argument", HX_ERR_UNSUPPORTED: "unsupported configuration",
                HX_ERR_LAUNCH: "CUDA launch failed",
                HX_ERR_SCRATCH_LIMIT: "request exceeds the fixed scratch size"}.get(rc, f"status {rc}")
        raise HelixError(f"{name}: {what}")
    return rc


def ptr(t):
    """Raw device pointer of a CUDA tensor (None -> NULL)."""
    if t is None:
        return None
    if not t.is_cuda:
        raise HelixError("helix KV kernels take CUDA tensors only (no CPU fallback)")
    return ctypes.c_void_p(t.data_ptr())


def stream(device=None):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise HelixError("helix KV kernels take CUDA tensors only (no CPU fallback)")


# ---- per-device error word and scratch -----------------------------------------

_err_words: dict = {}
_scratch: dict = {}


def err_word(device) -> torch.Tensor:
    dev = torch.device(device)
    key = dev.index if dev.index is not None else torch.cuda.current_device()
    w = _err_words.get(key)
    if w is None:
        w = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", key))
        _err_words[key] = w
    return w


def check_device_errors(device=None, reset: bool = True):
    """Synchronise and raise if any kernel flagged a device error."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    w = err_word(dev)
    torch.cuda.synchronize(dev)
    v = int(w.item())
    if v:
        if reset:
            w.zero_()
        msgs = [m for b, m in DEV_ERR.items() if v & b]
        raise HelixError("device error: " + ", ".join(msgs or [hex(v)]))


def scratch(device, name: str, nbytes: int) -> torch.Tensor:
    """Grow-only, zero-initialised byte buffer per (device, name).

    Kernels that count into scratch leave it zero on exit, so a buffer is
    zeroed once at allocation only.
    """
    dev = torch.device(device)
    key = (dev.index if dev.index is not None else torch.cuda.current_device(), name)
    buf = _scratch.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(max(int(nbytes), 256), dtype=torch.uint8, device=torch.device("cuda", key[0]))
        _scratch[key] = buf
    return buf


def version() -> str:
    return lib().hx_version().decode()
