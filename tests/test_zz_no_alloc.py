"""yn_moe_layer_noalloc (static device workspace) against yn_moe_layer.

Collected last so that it runs both alone and after every other GPU test in
the same process. Two calls in a row: the second one checks that the
combine counters at the front of the static workspace returned to zero.
"""
from __future__ import annotations

import ctypes as C

import pytest

torch = pytest.importorskip("torch")

from tests.gpu_helpers import REL_L2_TOL, DeviceModel, bf16_dev, bf16_np, hidden_rows, rel_l2, small_config
from yanah_b200 import _lib
from yanah_b200.device import stream_ptr

pytestmark = pytest.mark.gpu


def _noalloc(dm, layer, h_in, h_out):
    p = C.c_void_p()
    _lib.check(_lib.lib().yn_moe_layer_noalloc(C.byref(dm.dims), C.byref(dm.structs[layer]), h_in.data_ptr(),
                                               h_in.shape[0], None, 0, h_out.data_ptr(), stream_ptr(),
                                               C.byref(p)))
    return p.value


@pytest.mark.parametrize("bits,T", [(4, 1), (2, 3)])
def test_noalloc_matches_workspace_layer_twice(bits, T):
    cfg = small_config(bits=(bits,), hidden=2048, n_experts=512, top_k=10, inter=512, shared=512, seed=21)
    dm = DeviceModel(cfg)
    for call in range(2):
        h = bf16_dev(hidden_rows(cfg, T, stream=40 + call))
        ref = torch.empty_like(h)
        dm.layer(0, h, ref)
        got = torch.empty_like(h)
        scratch = _noalloc(dm, 0, h, got)
        torch.cuda.synchronize()
        code = C.c_int32(0)
        _lib.check(_lib.lib().yn_workspace_error(scratch, C.byref(dm.dims), stream_ptr(), C.byref(code)))
        assert code.value == 0
        err = rel_l2(bf16_np(got), bf16_np(ref))
        assert err < REL_L2_TOL, (call, err)


def test_noalloc_rejects_oversize_workspace():
    cfg = small_config(bits=(4,), hidden=2048, n_experts=512, top_k=10, inter=512, shared=512, seed=21)
    dm = DeviceModel(cfg)
    big = _lib.Dims(4096, 512, 16, 2048, 2048, 1, 1e-6)
    lib = _lib.lib()
    assert lib.yn_workspace_bytes(C.byref(big)) > (1 << 20)
    h = bf16_dev(hidden_rows(cfg, 1, stream=1))
    out = torch.empty_like(h)
    rc = lib.yn_moe_layer_noalloc(C.byref(big), C.byref(dm.structs[0]), h.data_ptr(), 1, None, 0, out.data_ptr(),
                                  stream_ptr(), None)
    assert rc == _lib.YN_E_UNSUPPORTED
    assert b"static scratch" in lib.yn_last_error()
