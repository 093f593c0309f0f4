"""ctypes binding of libyanah_b200.so (the C ABI in include/yanah_b200.h).

The library is built in-tree (``python -m yanah_b200.build``). There is no
fallback: if the shared object is missing or does not load, ``lib()`` raises.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libyanah_b200.so"

YN_OK, YN_E_INVALID, YN_E_UNSUPPORTED, YN_E_CUDA, YN_E_DEVICE = 0, -1, -2, -3, -4
YN_MAX_ROWS = 8
YN_MAX_TARGETS = 2
YN_NOALLOC_SCRATCH_BYTES = 1 << 20  # static workspace of yn_moe_layer_noalloc, per device


class YanahError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"yanah_b200 error {code}: {msg}")
        self.code = code


class QMat(C.Structure):
    _fields_ = [("weight", C.c_void_p), ("scales", C.c_void_p), ("biases", C.c_void_p),
                ("rows", C.c_int32), ("cols", C.c_int32), ("bits", C.c_int32), ("group_size", C.c_int32)]


class Dims(C.Structure):
    _fields_ = [("hidden", C.c_int32), ("n_experts", C.c_int32), ("top_k", C.c_int32),
                ("moe_inter", C.c_int32), ("shared_inter", C.c_int32), ("norm_topk", C.c_int32),
                ("rms_eps", C.c_float)]


class Record(C.Structure):
    _fields_ = [("bits", C.c_int32), ("group_size", C.c_int32), ("piece_offset", C.c_int64 * 9),
                ("record_bytes", C.c_int64)]


class Layer(C.Structure):
    _fields_ = [("post_norm", C.c_void_p), ("router", QMat), ("router_bias", C.c_void_p),
                ("shared_gate", QMat), ("shared_up", QMat), ("shared_down", QMat),
                ("shared_expert_gate", QMat), ("expert_base", C.c_void_p), ("slot_stride", C.c_int64),
                ("n_slots", C.c_int32), ("expert_slot", C.c_void_p), ("record", Record)]


class WsView(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("x", "logits", "ids", "weights", "flogits", "fprobs", "act",
                                          "act_sh", "sgate", "y", "y_shared", "error")]


class EpConfig(C.Structure):
    _fields_ = [("rank", C.c_int32), ("n_ranks", C.c_int32), ("rows_per_rank", C.c_int32),
                ("expert_lo", C.c_int32), ("expert_hi", C.c_int32), ("n_layers", C.c_int32)]


class EpLocalPtrs(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("x", "ids", "weights", "act_sh", "sgate", "y_shared", "error", "epoch")]


class EpSymPtrs(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("x_all", "ids_all", "y", "flags", "counter")]


YN_IPC_HANDLE_BYTES = 64

_P = C.c_void_p
_I = C.c_int32
_SIGS = {
    "yn_last_error": (C.c_char_p, []),
    "yn_version": (C.c_char_p, []),
    "yn_workspace_bytes": (C.c_size_t, [C.POINTER(Dims)]),
    "yn_workspace_init": (C.c_int, [_P, C.c_size_t, C.POINTER(Dims), _P]),
    "yn_workspace_error": (C.c_int, [_P, C.POINTER(Dims), _P, C.POINTER(C.c_int32)]),
    "yn_workspace_view": (C.c_int, [_P, C.POINTER(Dims), C.POINTER(WsView)]),
    "yn_dequantize": (C.c_int, [C.POINTER(QMat), _P, _P]),
    "yn_qlinear": (C.c_int, [C.POINTER(QMat), _P, _I, _P, _P]),
    "yn_route": (C.c_int, [_P, _I, C.POINTER(Dims), _P, _P, _P]),
    "yn_post_attention": (C.c_int, [C.POINTER(Dims), C.POINTER(Layer), _P, _I, C.POINTER(Layer), _I, _P, _P]),
    "yn_moe_up": (C.c_int, [C.POINTER(Dims), C.POINTER(Layer), _P, _P, _I, C.POINTER(C.c_int32), _I, _P, _P]),
    "yn_moe_down": (C.c_int, [C.POINTER(Dims), C.POINTER(Layer), _P, _P, _I, _P, _I, _P, _P, _P]),
    "yn_moe_layer": (C.c_int, [C.POINTER(Dims), C.POINTER(Layer), _P, _I, C.POINTER(Layer), _I, _P, _P, _P]),
    "yn_moe_layer_noalloc": (C.c_int, [C.POINTER(Dims), C.POINTER(Layer), _P, _I, C.POINTER(Layer), _I, _P, _P,
                                       C.POINTER(C.c_void_p)]),
    "yn_stack_table_bytes": (C.c_size_t, [_I]),
    "yn_stack_scratch_bytes": (C.c_size_t, [C.POINTER(Dims)]),
    "yn_stack_prepare": (C.c_int, [C.POINTER(Dims), C.POINTER(Layer), _I, _P, C.c_size_t]),
    "yn_stack_decode": (C.c_int, [C.POINTER(Dims), _P, C.POINTER(Layer), _I, _P, _I, _P, _P, C.c_size_t, _P, _P,
                                  _P, _P, _P]),
    "yn_stack_flow_scratch_bytes": (C.c_size_t, [C.POINTER(Dims)]),
    "yn_stack_flow_decode": (C.c_int, [C.POINTER(Dims), _P, C.POINTER(Layer), _I, _P, _I, _P, _P, C.c_size_t, _P,
                                       _P, _P, _P, _P]),
    "yn_stack_error": (C.c_int, [_P, C.POINTER(Dims), _P, C.POINTER(C.c_int32)]),
    "yn_rows_flow_scratch_bytes": (C.c_size_t, [C.POINTER(Dims), _I]),
    "yn_rows_flow_decode": (C.c_int, [C.POINTER(Dims), _P, C.POINTER(Layer), _I, _P, _I, _P, _P, C.c_size_t, _P,
                                      _P, _P, _P, _P]),
    "yn_slot_copy": (C.c_int, [_P, C.c_int64, C.POINTER(C.c_int32), C.POINTER(C.c_void_p), _I, C.c_int64, _P]),
    "yn_record_event": (C.c_int, [_P, _P]),
    "yn_event_create": (C.c_int, [C.POINTER(C.c_void_p)]),
    "yn_event_destroy": (C.c_int, [_P]),
    "yn_event_elapsed_ms": (C.c_int, [_P, _P, C.POINTER(C.c_float)]),
    "yn_synth_u32": (C.c_int, [_P, C.c_int64, C.c_uint64, C.c_uint64, _P]),
    "yn_synth_f16": (C.c_int, [_P, C.c_int64, C.c_uint64, C.c_uint64, C.c_float, _I, _P]),
    "yn_synth_bf16": (C.c_int, [_P, C.c_int64, C.c_uint64, C.c_uint64, C.c_float, C.c_float, _P]),
    "yn_ep_sym_bytes": (C.c_size_t, [C.POINTER(Dims), C.POINTER(EpConfig)]),
    "yn_ep_local_bytes": (C.c_size_t, [C.POINTER(Dims), C.POINTER(EpConfig)]),
    "yn_ep_init": (C.c_int, [_P, _P, C.POINTER(Dims), C.POINTER(EpConfig), _P]),
    "yn_ep_layer": (C.c_int, [C.POINTER(Dims), C.POINTER(Layer), _I, C.POINTER(EpConfig), _P, _P,
                              C.POINTER(C.c_void_p), _P, _P]),
    "yn_ep_step_end": (C.c_int, [_P, C.POINTER(Dims), C.POINTER(EpConfig), _P]),
    "yn_ep_error": (C.c_int, [_P, C.POINTER(Dims), C.POINTER(EpConfig), _P, C.POINTER(C.c_int32)]),
    "yn_ep_view": (C.c_int, [_P, C.POINTER(Dims), C.POINTER(EpConfig), C.POINTER(EpLocalPtrs)]),
    "yn_ep_sym_view": (C.c_int, [_P, C.POINTER(Dims), C.POINTER(EpConfig), C.POINTER(EpSymPtrs)]),
    "yn_device_alloc": (C.c_int, [C.c_size_t, C.POINTER(C.c_void_p)]),
    "yn_device_free": (C.c_int, [_P]),
    "yn_ipc_export": (C.c_int, [_P, _P]),
    "yn_ipc_import": (C.c_int, [_P, C.POINTER(C.c_void_p)]),
    "yn_ipc_close": (C.c_int, [_P]),
    "yn_memcpy": (C.c_int, [_P, _P, C.c_size_t, _P]),
    "yn_memcpy_async": (C.c_int, [_P, _P, C.c_size_t, _P]),
    "yn_rows_route_bytes": (C.c_size_t, [C.POINTER(Dims), _I]),
    "yn_rows_route": (C.c_int, [C.POINTER(Dims), C.POINTER(Layer), _P, _I, _P, _P, _P, _P, C.c_size_t, _P]),
    "yn_route_error": (C.c_int, [_P, C.POINTER(Dims), _P, C.POINTER(C.c_int32)]),
    "yn_to_f16_kperm": (C.c_int, [_P, C.c_int64, _I, _P, _P]),
    "yn_tc_experts": (C.c_int, [C.POINTER(Dims), C.POINTER(Layer), _I, _P, _I, _P, _P, C.c_int64, _P, _P, _P, _P]),
    "yn_gather_f16_kperm": (C.c_int, [_P, _P, C.c_int64, _I, _P, _P]),
    "yn_prefill_max_tiles": (C.c_int, [C.POINTER(Dims), _I, C.POINTER(C.c_int32), C.POINTER(C.c_int32)]),
    "yn_prefill_plan": (C.c_int, [C.POINTER(Dims), _P, _I, _P, _P, _P, _I, _P, _I, _P, _P, _P]),
    "yn_pairs_combine": (C.c_int, [C.POINTER(Dims), _P, _P, _P, _P, _P, _I, _P, _P]),
    "yn_gather_kperm": (C.c_int, [_P, _P, C.c_int64, _I, _I, _I, _P, _P]),
    "yn_scale_rows": (C.c_int, [_P, _P, C.c_int64, _I, _P, _P]),
    "yn_rows_route_shared": (C.c_int, [C.POINTER(Dims), _I, _P, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p)]),
}

_lib = None


def exported_symbols():
    """Names of the C entry points this binding expects (declared in the header)."""
    return sorted(_SIGS)


def lib() -> C.CDLL:
    """Load libyanah_b200.so (once). Raises if it is missing: there is no fallback."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is missing; build it with `python -m yanah_b200.build`")
        dll = C.CDLL(str(LIB_PATH), mode=os.RTLD_NOW | os.RTLD_GLOBAL)
        for name, (res, args) in _SIGS.items():
            f = getattr(dll, name)
            f.restype = res
            f.argtypes = args
        _lib = dll
    return _lib


def check(rc: int) -> None:
    if rc != YN_OK:
        msg = lib().yn_last_error().decode(errors="replace")
        raise YanahError(rc, msg)
