"""yn_moe_layer_noalloc (static device workspace) against yn_moe_layer.

yn_moe_layer_noalloc exists for callers that cannot hand the library a
device workspace: an FFI binding (cgo, JNI, ctypes) that owns no device
allocator, or a process whose free HBM has all gone to the expert slot pool.
It runs the same kernels as yn_moe_layer on the same inputs, so its outputs
must equal yn_moe_layer's bit for bit.

Collected last so that it runs both alone and after every other GPU test in
the same process. Calls in a row check that the combine counters at the
front of the shared static workspace return to zero after each call, also
when a call's counter region grows past the previous call's (a larger hidden
size) or shrinks below it.
"""
from __future__ import annotations

import ctypes as C

import pytest

torch = pytest.importorskip("torch")

from tests.gpu_helpers import DeviceModel, bf16_dev, hidden_rows, small_config
from yanah_b200 import _lib
from yanah_b200.device import stream_ptr

pytestmark = pytest.mark.gpu


def _noalloc(dm, layer, h_in, h_out):
    p = C.c_void_p()
    _lib.check(_lib.lib().yn_moe_layer_noalloc(C.byref(dm.dims), C.byref(dm.structs[layer]), h_in.data_ptr(),
                                               h_in.shape[0], None, 0, h_out.data_ptr(), stream_ptr(),
                                               C.byref(p)))
    return p.value


def _check_call(dm, T, stream_id):
    """One yn_moe_layer_noalloc call compared bit for bit with yn_moe_layer;
    the static workspace's error word must stay clear."""
    h = bf16_dev(hidden_rows(dm.cfg, T, stream=stream_id))
    ref = torch.empty_like(h)
    dm.layer(0, h, ref)
    got = torch.empty_like(h)
    scratch = _noalloc(dm, 0, h, got)
    torch.cuda.synchronize()
    code = C.c_int32(0)
    _lib.check(_lib.lib().yn_workspace_error(scratch, C.byref(dm.dims), stream_ptr(), C.byref(code)))
    assert code.value == 0
    assert torch.equal(got.view(torch.int16), ref.view(torch.int16)), stream_id
    return h, got


@pytest.mark.parametrize("bits,T", [(4, 1), (2, 3)])
def test_noalloc_matches_workspace_layer_twice(bits, T):
    cfg = small_config(bits=(bits,), hidden=2048, n_experts=512, top_k=10, inter=512, shared=512, seed=21)
    dm = DeviceModel(cfg)
    for call in range(2):
        _check_call(dm, T, 40 + call)


def test_noalloc_allocates_nothing():
    """After a warm-up call (module loading, first-use set-up), a call changes
    neither torch's allocator nor the device's free memory."""
    cfg = small_config(bits=(4,), hidden=2048, n_experts=512, top_k=10, inter=512, shared=512, seed=22)
    dm = DeviceModel(cfg)
    h = bf16_dev(hidden_rows(cfg, 2, stream=50))
    out = torch.empty_like(h)
    _noalloc(dm, 0, h, out)
    torch.cuda.synchronize()
    alloc0, free0 = torch.cuda.memory_allocated(), torch.cuda.mem_get_info()[0]
    _noalloc(dm, 0, h, out)
    torch.cuda.synchronize()
    assert torch.cuda.memory_allocated() == alloc0
    assert torch.cuda.mem_get_info()[0] == free0


def test_noalloc_counter_region_grows_and_shrinks():
    """hidden 2048, then 256 (smaller counter region), 2048 again (the region
    grows past the last call's: its extension is zeroed first), then 4096
    (larger than every earlier call, still inside the 1 MiB array)."""
    lib = _lib.lib()
    models = {}
    for H in (2048, 256, 4096):
        big = H == 2048
        cfg = small_config(bits=(4,), hidden=H, n_experts=512 if big else 64, top_k=10 if big else 4,
                           inter=512 if big else 256, shared=512 if big else 256, seed=23)
        models[H] = DeviceModel(cfg)
        assert lib.yn_workspace_bytes(C.byref(models[H].dims)) <= _lib.YN_NOALLOC_SCRATCH_BYTES
    for i, H in enumerate((2048, 256, 2048, 4096, 256)):
        _check_call(models[H], 2, 60 + i)


def test_noalloc_rejects_oversize_workspace():
    cfg = small_config(bits=(4,), hidden=2048, n_experts=512, top_k=10, inter=512, shared=512, seed=21)
    dm = DeviceModel(cfg)
    big = _lib.Dims(4096, 512, 16, 2048, 2048, 1, 1e-6)
    lib = _lib.lib()
    assert lib.yn_workspace_bytes(C.byref(big)) > _lib.YN_NOALLOC_SCRATCH_BYTES
    h = bf16_dev(hidden_rows(cfg, 1, stream=1))
    out = torch.empty_like(h)
    rc = lib.yn_moe_layer_noalloc(C.byref(big), C.byref(dm.structs[0]), h.data_ptr(), 1, None, 0, out.data_ptr(),
                                  stream_ptr(), None)
    assert rc == _lib.YN_E_UNSUPPORTED
    assert b"static scratch" in lib.yn_last_error()
