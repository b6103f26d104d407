"""lsx_readout_margin_fixed: the readout margin with the library's fixed device
scratch instead of a caller workspace, for callers that cannot allocate device
memory when they validate.  It must give what lsx_readout_margin_device gives on
the same inputs, call after call (and what the oracle gives), make no device
allocation, report non-finite scores through lsx_readout_status, and reject
sizes beyond its scratch.  Collected last so it also runs after every other test
has used the device."""
import ctypes as C

import numpy as np
import pytest

from laplacesscissors_b200 import synth
from laplacesscissors_b200._lib import BF16, F32, LsxError, check, lib

pytestmark = pytest.mark.gpu

SCRATCH = 4 << 20  # the fixed scratch per device


def _align(x):
    return (x + 255) & ~255


def bf16_need(rows):
    """Scratch bytes of a bf16-row call without an edit: the two status words, then
    per row a best-other key (8 B) and a target logit (4 B), each area 256-byte
    aligned."""
    return 256 + _align(rows * 8) + _align(rows * 4)


def _device_outputs(torch, dev, rows):
    return (torch.empty(rows, dtype=torch.float64, device=dev), torch.empty(rows, dtype=torch.int32, device=dev),
            torch.empty(rows, dtype=torch.float32, device=dev))


def _ptrs(outs):
    return [C.c_void_p(t.data_ptr()) for t in outs]


def _host(outs):
    return [t.cpu().numpy() for t in outs]


def _workspace_call(torch, gpu, weight, bias, V, H, hidden, hk, n, targets):
    dev = f"cuda:{gpu.device}"
    ws_bytes = lib.lsx_readout_workspace_bytes(V, H, n, None)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    ref = _device_outputs(torch, dev, n)
    check(lib.lsx_readout_margin_device(gpu.handle, weight.handle, bias.handle if bias else None, V, H,
                                        C.c_void_p(hidden.data_ptr()), hk, n, C.c_void_p(targets.data_ptr()), None,
                                        *_ptrs(ref), C.c_void_p(ws.data_ptr()), ws_bytes))
    check(lib.lsx_readout_status(gpu.handle, C.c_void_p(ws.data_ptr())))
    return _host(ref)


def _fixed_call(torch, gpu, weight, bias, V, H, hidden, hk, n, targets):
    """Enqueues the fixed-scratch call on the library's stream; the caller reads the
    outputs only after lsx_readout_status (which waits for that stream)."""
    out = _device_outputs(torch, f"cuda:{gpu.device}", n)
    check(lib.lsx_readout_margin_fixed(gpu.handle, weight.handle, bias.handle if bias else None, V, H,
                                       C.c_void_p(hidden.data_ptr()), hk, n, C.c_void_p(targets.data_ptr()),
                                       *_ptrs(out)))
    return out


@pytest.mark.parametrize("kind", ["bf16", "f32", "f32_bias"])
def test_fixed_scratch_matches_workspace_entry(gpu, kind):
    import torch
    V, H, n = 4099, 1024, 257 if kind == "bf16" else 200
    dev = f"cuda:{gpu.device}"
    w = synth.normal_bf16(3, 0, V * H, 0.02)
    weight = gpu.upload_raw(w, BF16)
    bias = gpu.upload_f32(synth.normal_f32(5, 10, V, 0.5)) if kind == "f32_bias" else None
    if kind == "bf16":
        hidden = torch.from_numpy(synth.readout_hidden(3, n, H).view(np.int16).copy()).to(dev)
        hk = BF16
    else:
        hidden = torch.from_numpy(synth.normal_f32(5, 9, n * H)).to(dev)
        hk = F32
    targets = torch.from_numpy(synth.readout_targets(3, n, V).astype(np.int32)).to(dev)
    m_ref, a_ref, t_ref = _workspace_call(torch, gpu, weight, bias, V, H, hidden, hk, n, targets)
    for call in range(2):
        torch.cuda.synchronize(dev)
        if call == 1:
            free_before = torch.cuda.mem_get_info(dev)[0]
        out = _fixed_call(torch, gpu, weight, bias, V, H, hidden, hk, n, targets)
        check(lib.lsx_readout_status(gpu.handle, None))
        gpu.synchronize()
        if call == 1:
            # the outputs were allocated before the measurement: the call itself allocates nothing
            assert torch.cuda.mem_get_info(dev)[0] == free_before
        m, a, t = _host(out)
        # Same kernels on the same inputs: the tolerance only allows for the order
        # of the atomic best-other reduction, which cannot change the maximum.
        assert np.array_equal(a, a_ref)
        np.testing.assert_allclose(m, m_ref, rtol=0, atol=1e-6)
        np.testing.assert_allclose(t, t_ref, rtol=0, atol=1e-6)


def test_fixed_scratch_matches_oracle(gpu, oracle):
    """A direct check against the oracle's readout on a small shape: argmax equal
    away from near-ties, margins within the readout tests' tolerance."""
    import torch
    V, H, n = 2053, 256, 131
    dev = f"cuda:{gpu.device}"
    w = synth.normal_bf16(4, 0, V * H, 0.02)
    rows = synth.readout_hidden(4, n, H)
    t_host = synth.readout_targets(4, n, V)
    weight = gpu.upload_raw(w, BF16)
    hidden = torch.from_numpy(rows.view(np.int16).copy()).to(dev)
    targets = torch.from_numpy(t_host.astype(np.int32)).to(dev)
    out = _fixed_call(torch, gpu, weight, None, V, H, hidden, BF16, n, targets)
    check(lib.lsx_readout_status(gpu.handle, None))
    m, a, t = _host(out)
    m_ref, a_ref, t_ref = oracle.readout_rows(w, oracle.BF16, None, V, H, synth.bf16_to_f32(rows), t_host)
    near = np.abs(m_ref) < 1e-3
    assert np.array_equal(a.view(np.uint32)[~near], a_ref[~near])
    assert np.all(np.abs(m - m_ref) <= 1e-5 * (1 + np.abs(m_ref)))
    assert np.all(np.abs(t.astype(np.float64) - t_ref) <= 1e-5 * (1 + np.abs(t_ref)))


def test_fixed_scratch_reports_nonfinite_scores(gpu):
    """A hidden row holding an infinity gives non-finite scores: the status read
    after the call says so (the reference rejects non-finite scores,
    src/model.rs:680-683), and the next clean call reports a clean status."""
    import torch
    V, H, n = 1031, 256, 64
    dev = f"cuda:{gpu.device}"
    weight = gpu.upload_raw(synth.normal_bf16(6, 0, V * H, 0.02), BF16)
    host = synth.normal_f32(6, 9, n * H).reshape(n, H)
    bad = host.copy()
    bad[17, 5] = np.inf
    targets = torch.from_numpy(synth.readout_targets(6, n, V).astype(np.int32)).to(dev)
    _fixed_call(torch, gpu, weight, None, V, H, torch.from_numpy(bad.reshape(-1)).to(dev), F32, n, targets)
    with pytest.raises(LsxError) as err:
        check(lib.lsx_readout_status(gpu.handle, None))
    assert err.value.status == 4  # LSX_E_NONFINITE
    _fixed_call(torch, gpu, weight, None, V, H, torch.from_numpy(host.reshape(-1)).to(dev), F32, n, targets)
    check(lib.lsx_readout_status(gpu.handle, None))


def test_fixed_scratch_size_boundary_bf16(gpu):
    """bf16 rows: the largest row count whose working set fits the scratch runs and
    matches the workspace entry; one row more is rejected before anything is
    enqueued."""
    import torch
    V, H = 1031, 128
    dev = f"cuda:{gpu.device}"
    rows = (SCRATCH - 256) // 12
    while bf16_need(rows) > SCRATCH:
        rows -= 1
    assert bf16_need(rows + 1) > SCRATCH
    weight = gpu.upload_raw(synth.normal_bf16(8, 0, V * H, 0.02), BF16)
    hidden = torch.from_numpy(synth.readout_hidden(8, rows + 1, H).view(np.int16).copy()).to(dev)
    targets = torch.from_numpy(synth.readout_targets(8, rows + 1, V).astype(np.int32)).to(dev)
    m_ref, a_ref, _ = _workspace_call(torch, gpu, weight, None, V, H, hidden, BF16, rows, targets)
    out = _fixed_call(torch, gpu, weight, None, V, H, hidden, BF16, rows, targets)
    check(lib.lsx_readout_status(gpu.handle, None))
    m, a, _ = _host(out)
    assert np.array_equal(a, a_ref)
    np.testing.assert_allclose(m, m_ref, rtol=0, atol=1e-6)
    with pytest.raises(LsxError, match="fixed scratch"):
        _fixed_call(torch, gpu, weight, None, V, H, hidden, BF16, rows + 1, targets)


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
    # sizes whose products would wrap are refused by the argument checks, not by the size test
    with pytest.raises(LsxError, match="row count|weight dimensions"):
        check(lib.lsx_readout_margin_fixed(gpu.handle, weight.handle, None, V, H, C.c_void_p(hidden.data_ptr()), F32,
                                           1 << 40, C.c_void_p(targets.data_ptr()), *_ptrs(out)))
