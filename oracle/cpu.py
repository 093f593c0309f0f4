"""ctypes wrapper of the C oracle (oracle/yn_oracle.c) — TEST INFRASTRUCTURE.

Gives numpy-level access to the CPU restatement: dequantisation, canonical
QuantizedLinear, RMSNorm, routing, lookahead softmax, SwiGLU experts, the
shared expert, the combine, and the bit-exact synthetic generator that
regenerates any expert record of a seeded stack on the CPU.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path
from typing import Dict, List, Optional, Sequence

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "libyn_oracle.so"


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


class QMat(C.Structure):
    _fields_ = [("w", C.c_void_p), ("s", C.c_void_p), ("b", C.c_void_p), ("rows", C.c_int32),
                ("cols", C.c_int32), ("bits", C.c_int32), ("gs", C.c_int32)]


class Dense(C.Structure):
    _fields_ = [("norm", C.c_void_p), ("router", QMat), ("rbias", C.c_void_p), ("sh_gate", QMat),
                ("sh_up", QMat), ("sh_down", QMat), ("sgate", QMat), ("has_shared", C.c_int32)]


class Dims(C.Structure):
    _fields_ = [("H", C.c_int32), ("E", C.c_int32), ("K", C.c_int32), ("I", C.c_int32), ("Ish", C.c_int32),
                ("norm_topk", C.c_int32), ("eps", C.c_float)]


class Record(C.Structure):
    _fields_ = [("bits", C.c_int32), ("gs", C.c_int32), ("off", C.c_int64 * 9)]


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        _lib = C.CDLL(str(LIB_PATH))
        P, I, I64, U64, F = C.c_void_p, C.c_int, C.c_int64, C.c_uint64, C.c_float
        sig = {
            "yo_synth_u32": [P, I64, U64, U64, I64],
            "yo_synth_f16": [P, I64, U64, U64, F, I, I64],
            "yo_synth_bf16": [P, I64, U64, U64, F, F, I64],
            "yo_f32_to_bf16": [P, I64, P], "yo_f32_to_f16": [P, I64, P], "yo_f16_to_f32": [P, I64, P],
            "yo_qlinear": [C.POINTER(QMat), P, I, P],
            "yo_dequantize": [C.POINTER(QMat), P],
            "yo_rmsnorm": [P, P, I, F, P],
            "yo_route_row": [P, I, I, I, P, P, P],
            "yo_route": [P, I, I, I, I, P, P],
            "yo_softmax_f32": [P, I, P],
            "yo_post_attention": [C.POINTER(Dims), C.POINTER(Dense), P, I, C.POINTER(Dense), I, P, P, P, P, P, P, P],
            "yo_expert": [C.POINTER(Dims), P, C.POINTER(Record), P, P, P],
            "yo_shared_down": [C.POINTER(Dims), C.POINTER(Dense), P, F, P],
            "yo_combine": [C.POINTER(Dims), P, P, P, P, I, P],
            "yo_set_threads": [I],
        }
        for name, args in sig.items():
            f = getattr(_lib, name)
            f.argtypes = args
            f.restype = None
        _lib.yo_expf.argtypes = [C.c_float]
        _lib.yo_expf.restype = C.c_float
        _lib.yo_num_threads.argtypes = []
        _lib.yo_num_threads.restype = C.c_int
    return _lib


def _p(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data


# ----------------------------------------------------------------- helpers
def synth_u32(n: int, seed: int, sid: int, start: int = 0) -> np.ndarray:
    out = np.empty(n, np.uint32)
    lib().yo_synth_u32(_p(out), n, seed, sid, start)
    return out


def synth_f16(n: int, seed: int, sid: int, std: float, absolute: bool, start: int = 0) -> np.ndarray:
    out = np.empty(n, np.uint16)
    lib().yo_synth_f16(_p(out), n, seed, sid, std, int(absolute), start)
    return out


def synth_bf16(n: int, seed: int, sid: int, std: float, mean: float = 0.0, start: int = 0) -> np.ndarray:
    out = np.empty(n, np.uint16)
    lib().yo_synth_bf16(_p(out), n, seed, sid, std, mean, start)
    return out


def qmat(w: np.ndarray, s: np.ndarray, b: np.ndarray, cols: int, bits: int, gs: int) -> QMat:
    s16 = np.ascontiguousarray(np.asarray(s, np.float16).view(np.uint16))
    b16 = np.ascontiguousarray(np.asarray(b, np.float16).view(np.uint16))
    w = np.ascontiguousarray(w, np.uint32)
    m = QMat(w.ctypes.data, s16.ctypes.data, b16.ctypes.data, w.shape[0], cols, bits, gs)
    m._keep = (w, s16, b16)
    return m


def dequantize(w, s, b, cols: int, bits: int, gs: int) -> np.ndarray:
    m = qmat(w, s, b, cols, bits, gs)
    out = np.empty((m.rows, cols), np.float32)
    lib().yo_dequantize(C.byref(m), _p(out))
    return out


def qlinear(w, s, b, cols: int, bits: int, gs: int, x_bf16: np.ndarray) -> np.ndarray:
    m = qmat(w, s, b, cols, bits, gs)
    x = np.ascontiguousarray(x_bf16, np.uint16).reshape(-1, cols)
    out = np.empty((x.shape[0], m.rows), np.float32)
    lib().yo_qlinear(C.byref(m), _p(x), x.shape[0], _p(out))
    return out


def rmsnorm(h_bf16: np.ndarray, w_bf16: np.ndarray, eps: float) -> np.ndarray:
    h = np.ascontiguousarray(h_bf16, np.uint16)
    out = np.empty_like(h)
    for t in range(h.shape[0]):
        lib().yo_rmsnorm(_p(h[t]), _p(np.ascontiguousarray(w_bf16, np.uint16)), h.shape[1], eps, _p(out[t]))
    return out


def route(logits: np.ndarray, k: int, norm: bool = True):
    lg = np.ascontiguousarray(logits, np.float32)
    T, E = lg.shape
    ids = np.empty((T, k), np.int32)
    w = np.empty((T, k), np.float32)
    lib().yo_route(_p(lg), T, E, k, int(norm), _p(ids), _p(w))
    return ids, w


def route_probs(logits_row: np.ndarray, k: int, norm: bool = True):
    lg = np.ascontiguousarray(logits_row, np.float32)
    E = lg.shape[0]
    ids, w, p = np.empty(k, np.int32), np.empty(k, np.float32), np.empty(E, np.float32)
    lib().yo_route_row(_p(lg), E, k, int(norm), _p(ids), _p(w), _p(p))
    return ids, w, p


def softmax_f32(logits_row: np.ndarray) -> np.ndarray:
    lg = np.ascontiguousarray(logits_row, np.float32)
    out = np.empty_like(lg)
    lib().yo_softmax_f32(_p(lg), lg.shape[0], _p(out))
    return out


def expf(x: float) -> float:
    return float(lib().yo_expf(float(x)))


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().yo_f32_to_bf16(_p(x), x.size, _p(out))
    return out


def f32_to_f16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().yo_f32_to_f16(_p(x), x.size, _p(out))
    return out


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


# ------------------------------------------------------------ whole layers
class OracleStack:
    """CPU restatement of a seeded synthetic stack (see yanah_b200.synthetic).

    Dense weights come from the same seeded numpy generator as the device
    copies; routed expert records are regenerated on demand with the
    bit-exact counter generator and cached per (layer, expert)."""

    def __init__(self, cfg, threads: int = 0):
        from yanah_b200.synthetic import dense_layer  # input specification only
        self.cfg = cfg
        if threads:
            lib().yo_set_threads(threads)
        self.dims = Dims(cfg.hidden, cfg.n_experts, cfg.top_k, cfg.moe_inter, cfg.shared_inter, int(cfg.norm_topk),
                         cfg.eps)
        self._dense = {}
        self._dense_np = {}
        self._records: Dict[tuple, np.ndarray] = {}
        self._dense_layer = dense_layer

    def dense(self, layer: int) -> Dense:
        if layer not in self._dense:
            cfg = self.cfg
            d = self._dense_layer(cfg, layer)
            H, g = cfg.hidden, cfg.dense_group
            D = Dense()
            norm = np.ascontiguousarray(d.norm)
            D.norm = norm.ctypes.data
            D.router = qmat(*d.router, H, 8, g)
            rb = np.ascontiguousarray(d.router_bias, np.float32)
            D.rbias = rb.ctypes.data
            keep = [norm, rb, D.router]
            if cfg.shared_inter:
                D.sh_gate = qmat(*d.shared_gate, H, 8, g)
                D.sh_up = qmat(*d.shared_up, H, 8, g)
                D.sh_down = qmat(*d.shared_down, cfg.shared_inter, 8, g)
                D.sgate = qmat(*d.shared_expert_gate, H, 8, g)
                D.has_shared = 1
                keep += [D.sh_gate, D.sh_up, D.sh_down, D.sgate]
            D._keep = keep
            self._dense[layer] = D
            self._dense_np[layer] = d
        return self._dense[layer]

    def dense_np(self, layer: int):
        self.dense(layer)
        return self._dense_np[layer]

    def record(self, layer: int, expert: int) -> np.ndarray:
        key = (layer, expert)
        r = self._records.get(key)
        if r is None:
            r = expert_record(self.cfg, layer, expert)
            self._records[key] = r
        return r

    def record_struct(self, layer: int) -> Record:
        spec = self.cfg.record_spec(layer)
        R = Record(spec.bits, spec.group_size)
        for i, o in enumerate(spec.offsets):
            R.off[i] = o
        return R

    def post_attention(self, layer: int, h1: np.ndarray, targets: Sequence[int] = ()):
        cfg = self.cfg
        h1 = np.ascontiguousarray(h1, np.uint16).reshape(-1, cfg.hidden)
        T, H, E, K = h1.shape[0], cfg.hidden, cfg.n_experts, cfg.top_k
        Ish = max(cfg.shared_inter, 1)
        out = dict(x=np.empty((T, H), np.uint16), logits=np.empty((T, E), np.float32),
                   act_sh=np.zeros((T, Ish), np.uint16), sgate=np.zeros(T, np.float32),
                   ids=np.empty((T, K), np.int32), w=np.empty((T, K), np.float32),
                   fprobs=np.zeros((max(len(targets), 1), E), np.float32))
        tg = (Dense * max(len(targets), 1))(*[self.dense(t) for t in targets]) if targets else None
        lib().yo_post_attention(C.byref(self.dims), C.byref(self.dense(layer)), _p(h1), T, tg, len(targets),
                                _p(out["x"]), _p(out["logits"]), _p(out["act_sh"]), _p(out["sgate"]),
                                _p(out["ids"]), _p(out["w"]), _p(out["fprobs"]))
        return out

    def expert(self, layer: int, expert: int, x_row: np.ndarray):
        cfg = self.cfg
        rec = self.record(layer, expert)
        R = self.record_struct(layer)
        act = np.empty(cfg.moe_inter, np.uint16)
        y = np.empty(cfg.hidden, np.uint16)
        x = np.ascontiguousarray(x_row, np.uint16)
        lib().yo_expert(C.byref(self.dims), _p(rec), C.byref(R), _p(x), _p(act), _p(y))
        return act, y

    def shared_down(self, layer: int, act_sh_row: np.ndarray, sg: float) -> np.ndarray:
        y = np.empty(self.cfg.hidden, np.uint16)
        a = np.ascontiguousarray(act_sh_row, np.uint16)
        lib().yo_shared_down(C.byref(self.dims), C.byref(self.dense(layer)), _p(a), float(sg), _p(y))
        return y

    def combine(self, y: np.ndarray, w: np.ndarray, ysh: Optional[np.ndarray], h_res: Optional[np.ndarray],
                mode: int) -> np.ndarray:
        out = np.empty(self.cfg.hidden, np.uint16)
        y = np.ascontiguousarray(y, np.uint16)
        w = np.ascontiguousarray(w, np.float32)
        ysh = None if ysh is None else np.ascontiguousarray(ysh, np.uint16)
        h_res = None if h_res is None else np.ascontiguousarray(h_res, np.uint16)
        lib().yo_combine(C.byref(self.dims), _p(y), _p(w), _p(ysh), _p(h_res), mode, _p(out))
        return out

    def layer(self, layer: int, h1: np.ndarray, targets: Sequence[int] = (), mode: int = 2):
        """Whole layer for T rows; returns the post-attention dict plus act/y/ysh/out."""
        cfg = self.cfg
        h1 = np.ascontiguousarray(h1, np.uint16).reshape(-1, cfg.hidden)
        pa = self.post_attention(layer, h1, targets)
        T, K = h1.shape[0], cfg.top_k
        act = np.empty((T, K, cfg.moe_inter), np.uint16)
        y = np.empty((T, K, cfg.hidden), np.uint16)
        ysh = np.zeros((T, cfg.hidden), np.uint16)
        out = np.empty((T, cfg.hidden), np.uint16)
        for t in range(T):
            for j in range(K):
                act[t, j], y[t, j] = self.expert(layer, int(pa["ids"][t, j]), pa["x"][t])
            sh = mode >= 1 and cfg.shared_inter > 0
            if sh:
                ysh[t] = self.shared_down(layer, pa["act_sh"][t], pa["sgate"][t])
            out[t] = self.combine(y[t], pa["w"][t], ysh[t] if sh else None, h1[t], mode)
        pa.update(act=act, y=y, ysh=ysh, out=out)
        return pa


def expert_record(cfg, layer: int, expert: int) -> np.ndarray:
    """The seeded record of (layer, expert) as bytes, generated on the CPU."""
    from yanah_b200.synthetic import EXPERT_BIAS_STD, EXPERT_SCALE_STD, expert_stream_id, piece_elements
    spec = cfg.record_spec(layer)
    parts = []
    for p, piece in enumerate(spec.pieces):
        n = piece_elements(spec, p)
        sid = expert_stream_id(layer, p)
        if piece.dtype == "U32":
            a = synth_u32(n, cfg.seed, sid, start=expert * n)
        else:
            scale = p % 3 == 1
            a = synth_f16(n, cfg.seed, sid, EXPERT_SCALE_STD if scale else EXPERT_BIAS_STD, scale, start=expert * n)
        parts.append(a.view(np.uint8))
    return np.concatenate(parts)
