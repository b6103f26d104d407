"""lsx_readout_margin_fixed: the readout margin with the library's fixed device
scratch instead of a caller workspace.  It must give what lsx_readout_margin_device
gives on the same inputs, call after call, make no device allocation, and reject
sizes beyond its scratch.  Collected last so it also runs after every other test
has used the device."""
import ctypes as C

import numpy as np
import pytest

from laplacesscissors_b200 import synth
from laplacesscissors_b200._lib import BF16, F32, LsxError, check, lib

pytestmark = pytest.mark.gpu


def _device_outputs(torch, dev, rows):
    return (torch.empty(rows, dtype=torch.float64, device=dev), torch.empty(rows, dtype=torch.int32, device=dev),
            torch.empty(rows, dtype=torch.float32, device=dev))


def _ptrs(outs):
    return [C.c_void_p(t.data_ptr()) for t in outs]


def _host(outs):
    return [t.cpu().numpy() for t in outs]


@pytest.mark.parametrize("kind", ["bf16", "f32"])
def test_fixed_scratch_matches_workspace_entry(gpu, kind):
    import torch
    V, H, n = 4099, 1024, 257 if kind == "bf16" else 200
    dev = f"cuda:{gpu.device}"
    w = synth.normal_bf16(3, 0, V * H, 0.02)
    weight = gpu.upload_raw(w, BF16)
    if kind == "bf16":
        hidden = torch.from_numpy(synth.readout_hidden(3, n, H).view(np.int16).copy()).to(dev)
        hk = BF16
    else:
        hidden = torch.from_numpy(synth.normal_f32(5, 9, n * H)).to(dev)
        hk = F32
    targets = torch.from_numpy(synth.readout_targets(3, n, V).astype(np.int32)).to(dev)
    ws_bytes = lib.lsx_readout_workspace_bytes(V, H, n, None)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    ref = _device_outputs(torch, dev, n)
    check(lib.lsx_readout_margin_device(gpu.handle, weight.handle, None, V, H, C.c_void_p(hidden.data_ptr()), hk, n,
                                        C.c_void_p(targets.data_ptr()), None, *_ptrs(ref), C.c_void_p(ws.data_ptr()),
                                        ws_bytes))
    gpu.synchronize()
    m_ref, a_ref, t_ref = _host(ref)
    for call in range(2):
        out = _device_outputs(torch, dev, n)
        torch.cuda.synchronize(dev)
        if call == 1:
            free_before = torch.cuda.mem_get_info(dev)[0]
        check(lib.lsx_readout_margin_fixed(gpu.handle, weight.handle, None, V, H, C.c_void_p(hidden.data_ptr()), hk,
                                           n, C.c_void_p(targets.data_ptr()), *_ptrs(out)))
        gpu.synchronize()
        if call == 1:
            assert torch.cuda.mem_get_info(dev)[0] == free_before
        m, a, t = _host(out)
        # Same kernels on the same inputs: the tolerance only allows for the order
        # of the atomic best-other reduction, which cannot change the maximum.
        assert np.array_equal(a, a_ref)
        np.testing.assert_allclose(m, m_ref, rtol=0, atol=1e-6)
        np.testing.assert_allclose(t, t_ref, rtol=0, atol=1e-6)


def test_fixed_scratch_rejects_oversized_calls(gpu):
    import torch
    V, H = 4099, 1024
    dev = f"cuda:{gpu.device}"
    weight = gpu.upload_raw(synth.normal_bf16(3, 0, V * H, 0.02), BF16)
    rows = 2048  # F32 hidden: 2048 x 4 KiB of bf16 hi/lo planes alone exceed 4 MiB
    hidden = torch.zeros(rows * H, dtype=torch.float32, device=dev)
    targets = torch.zeros(rows, dtype=torch.int32, device=dev)
    out = _device_outputs(torch, dev, rows)
    with pytest.raises(LsxError, match="fixed scratch"):
        check(lib.lsx_readout_margin_fixed(gpu.handle, weight.handle, None, V, H, C.c_void_p(hidden.data_ptr()), F32,
                                           rows, C.c_void_p(targets.data_ptr()), *_ptrs(out)))
