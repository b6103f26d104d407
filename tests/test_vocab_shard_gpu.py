"""Vocabulary-sharded readout validation on one GPU.  The lm_head is split into
uneven row blocks; each block is scored by lsx_readout_shard_device, the
partials are max-merged on the device and finalised by lsx_readout_merge_device.
Every logit is the same dot product whichever block it falls in, so margins,
first argmaxes and target logits must equal the unsharded
lsx_readout_margin_device bit for bit (tie rules of src/diagnosis.rs:58-80)."""
import ctypes as C

import numpy as np
import pytest

import laplacesscissors_b200 as lsx
from laplacesscissors_b200 import DeviceRotation, ReadoutRotation, synth
from laplacesscissors_b200._lib import BF16, F32, check, lib
from laplacesscissors_b200.sharding import vocab_sharded_margin

pytestmark = pytest.mark.gpu

FLIP = -(1 << 63)


def device_inputs(gpu, hidden, targets):
    import torch
    dev = torch.device("cuda", gpu.device)
    h = torch.from_numpy(np.ascontiguousarray(hidden)).to(dev)
    t = torch.from_numpy(np.ascontiguousarray(targets, dtype=np.uint32).view(np.int32)).to(dev)
    return h, t


def unsharded(gpu, w, bias, V, H, h, kind, t, rot):
    import torch
    n = t.numel()
    r = rot.handle if rot else None
    ws = torch.empty(lib.lsx_readout_workspace_bytes(V, H, n, r), dtype=torch.uint8, device=h.device)
    margin = torch.empty(n, dtype=torch.float64, device=h.device)
    amax = torch.empty(n, dtype=torch.int32, device=h.device)
    tl = torch.empty(n, dtype=torch.float32, device=h.device)
    weight = gpu.upload_raw(w, BF16)
    b = gpu.upload_f32(bias) if bias is not None else None
    torch.cuda.synchronize(h.device)
    check(lib.lsx_readout_margin_device(gpu.handle, weight.handle, b.handle if b else None, V, H,
                                        C.c_void_p(h.data_ptr()), kind, n, C.c_void_p(t.data_ptr()), r,
                                        C.c_void_p(margin.data_ptr()), C.c_void_p(amax.data_ptr()),
                                        C.c_void_p(tl.data_ptr()), C.c_void_p(ws.data_ptr()), ws.numel()))
    gpu.synchronize()
    return margin.cpu().numpy(), amax.cpu().numpy().view(np.uint32), tl.cpu().numpy()


def sharded(gpu, w, bias, V, H, h, kind, t, rot, bounds):
    import torch
    n = t.numel()
    r = rot.handle if rot else None
    w2 = w.reshape(V, H)
    keys, tlogs, keep = [], [], []
    for v0, v1 in bounds:
        ws_shard = gpu.upload_raw(np.ascontiguousarray(w2[v0:v1]), BF16)
        b_shard = gpu.upload_f32(bias[v0:v1]) if bias is not None else None
        ws = torch.empty(lib.lsx_readout_workspace_bytes(v1 - v0, H, n, r), dtype=torch.uint8, device=h.device)
        k = torch.empty(n, dtype=torch.int64, device=h.device)
        tl = torch.empty(n, dtype=torch.float32, device=h.device)
        torch.cuda.synchronize(h.device)
        check(lib.lsx_readout_shard_device(gpu.handle, ws_shard.handle, b_shard.handle if b_shard else None, v0,
                                           v1 - v0, H, C.c_void_p(h.data_ptr()), kind, n, C.c_void_p(t.data_ptr()),
                                           r, C.c_void_p(k.data_ptr()), C.c_void_p(tl.data_ptr()),
                                           C.c_void_p(ws.data_ptr()), ws.numel()))
        gpu.synchronize()
        keys.append(k ^ FLIP)
        tlogs.append(tl)
        keep.append((ws_shard, b_shard, ws))
    key = torch.stack(keys).max(dim=0).values ^ FLIP
    tlog = torch.stack(tlogs).max(dim=0).values
    margin = torch.empty(n, dtype=torch.float64, device=h.device)
    amax = torch.empty(n, dtype=torch.int32, device=h.device)
    tl = torch.empty(n, dtype=torch.float32, device=h.device)
    torch.cuda.synchronize(h.device)
    check(lib.lsx_readout_merge_device(gpu.handle, C.c_void_p(key.data_ptr()), C.c_void_p(tlog.data_ptr()),
                                       C.c_void_p(t.data_ptr()), n, C.c_void_p(margin.data_ptr()),
                                       C.c_void_p(amax.data_ptr()), C.c_void_p(tl.data_ptr())))
    gpu.synchronize()
    return margin.cpu().numpy(), amax.cpu().numpy().view(np.uint32), tl.cpu().numpy()


def edit_of(kind, H):
    if kind == "plane":
        rng = np.random.default_rng(1)
        u = rng.standard_normal(H)
        u /= np.linalg.norm(u)
        v = rng.standard_normal(H)
        v -= (v @ u) * u
        v /= np.linalg.norm(v)
        return ReadoutRotation(u, v, 0.35)
    if kind == "joint":
        return lsx.random_subspace_rotation(H, 16, 3.0, seed=4)
    return None


@pytest.mark.parametrize("hidden_kind,edit,with_bias", [("bf16", None, False), ("f32", None, True),
                                                        ("bf16", "joint", False), ("f32", "plane", True)])
def test_vocab_shards_equal_unsharded(gpu, hidden_kind, edit, with_bias):
    V, H, n = 3001, 256, 300
    w = synth.normal_bf16(3, 0, V * H, 0.02)
    targets = synth.readout_targets(3, n, V)
    targets[:3] = [0, 1001, V - 1]  # first row, a two-row shard, last row
    if hidden_kind == "bf16":
        hidden, kind = synth.readout_hidden(3, n, H), BF16
    else:
        hidden, kind = synth.normal_f32(5, 9, n * H).reshape(n, H), F32
    bias = synth.normal_f32(5, 10, V, 0.5) if with_bias else None
    spec = edit_of(edit, H)
    rot = DeviceRotation.upload_edit(gpu, spec, H) if spec else None
    h, t = device_inputs(gpu, hidden, targets)
    ref = unsharded(gpu, w, bias, V, H, h, kind, t, rot)
    got = sharded(gpu, w, bias, V, H, h, kind, t, rot, [(0, 1000), (1000, 1002), (1002, V)])
    for a, b in zip(got, ref):
        assert np.array_equal(a, b), np.nonzero(a != b)[0][:8]


def test_sharded_entry_single_rank(gpu):
    """vocab_sharded_margin with one rank (no process group) is the whole readout."""
    V, H, n = 2053, 128, 130
    w = synth.normal_bf16(7, 0, V * H, 0.02)
    hidden = synth.readout_hidden(7, n, H)
    targets = synth.readout_targets(7, n, V)
    h, t = device_inputs(gpu, hidden, targets)
    ref = unsharded(gpu, w, None, V, H, h, BF16, t, None)
    weight = gpu.upload_raw(w, BF16)
    margin, amax, tl = vocab_sharded_margin(gpu, weight, None, 0, V, H, h.data_ptr(), BF16, n, t.data_ptr())
    gpu.synchronize()
    got = (margin.cpu().numpy(), amax.cpu().numpy().view(np.uint32), tl.cpu().numpy())
    for a, b in zip(got, ref):
        assert np.array_equal(a, b)


@pytest.mark.parametrize("hidden_kind,edit", [("bf16", None), ("f32", "joint")])
def test_packed_partials_equal_unsharded(gpu, hidden_kind, edit):
    """lsx_readout_partials_device per shard, an element-wise signed maximum of the
    packed int64 partials (what one all-reduce MAX computes across ranks), then
    lsx_readout_partials_merge_device: equal to the unsharded readout bit for bit."""
    import torch
    V, H, n = 3001, 256, 300
    w = synth.normal_bf16(3, 0, V * H, 0.02)
    targets = synth.readout_targets(3, n, V)
    targets[:3] = [0, 1001, V - 1]
    if hidden_kind == "bf16":
        hidden, kind = synth.readout_hidden(3, n, H), BF16
    else:
        hidden, kind = synth.normal_f32(5, 9, n * H).reshape(n, H), F32
    spec = edit_of(edit, H)
    rot = DeviceRotation.upload_edit(gpu, spec, H) if spec else None
    r = rot.handle if rot else None
    h, t = device_inputs(gpu, hidden, targets)
    ref = unsharded(gpu, w, None, V, H, h, kind, t, rot)
    w2 = w.reshape(V, H)
    merged, keep = None, []
    for v0, v1 in [(0, 1000), (1000, 1002), (1002, V)]:
        shard = gpu.upload_raw(np.ascontiguousarray(w2[v0:v1]), BF16)
        ws = torch.empty(lib.lsx_readout_workspace_bytes(v1 - v0, H, n, r), dtype=torch.uint8, device=h.device)
        part = torch.empty(2 * n, dtype=torch.int64, device=h.device)
        torch.cuda.synchronize(h.device)
        check(lib.lsx_readout_partials_device(gpu.handle, shard.handle, None, v0, v1 - v0, H,
                                              C.c_void_p(h.data_ptr()), kind, n, C.c_void_p(t.data_ptr()), r,
                                              C.c_void_p(part.data_ptr()), C.c_void_p(ws.data_ptr()), ws.numel()))
        check(lib.lsx_readout_status(gpu.handle, C.c_void_p(ws.data_ptr())))
        merged = part if merged is None else torch.maximum(merged, part)
        keep.append((shard, ws))
    margin = torch.empty(n, dtype=torch.float64, device=h.device)
    amax = torch.empty(n, dtype=torch.int32, device=h.device)
    tl = torch.empty(n, dtype=torch.float32, device=h.device)
    torch.cuda.synchronize(h.device)
    check(lib.lsx_readout_partials_merge_device(gpu.handle, C.c_void_p(merged.data_ptr()), C.c_void_p(t.data_ptr()),
                                                n, C.c_void_p(margin.data_ptr()), C.c_void_p(amax.data_ptr()),
                                                C.c_void_p(tl.data_ptr())))
    gpu.synchronize()
    got = (margin.cpu().numpy(), amax.cpu().numpy().view(np.uint32), tl.cpu().numpy())
    for a, b in zip(got, ref):
        assert np.array_equal(a, b), np.nonzero(a != b)[0][:8]
