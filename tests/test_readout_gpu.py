"""Fused readout-margin validation (tcgen05 kernel) against the oracle:
margins within tolerance, argmax bit-exact except at near-ties (|margin| < 1e-3),
over odd shapes, bf16 and f32 hidden states, plane and joint edits, and the
readout-validation workload at full size on a sample of rows."""
import numpy as np
import pytest

import laplacesscissors_b200 as lsx
from conftest import GOLDEN
from laplacesscissors_b200 import DeviceRotation, ReadoutRotation, diagnosis, synth
from laplacesscissors_b200._lib import BF16

pytestmark = pytest.mark.gpu


def check_rows(margin, amax, tl, ref, tol=2e-3):
    m_ref, a_ref, t_ref = ref
    near = np.abs(m_ref) < 1e-3
    assert np.all(np.isfinite(margin))
    assert np.array_equal(amax[~near], a_ref[~near]), np.nonzero(amax != a_ref)[0][:8]
    assert np.all(np.abs(margin - m_ref) <= tol * (1 + np.abs(m_ref)))
    assert np.all(np.abs(tl.astype(np.float64) - t_ref) <= tol * (1 + np.abs(t_ref)))


def problem(V, H, n, seed=3, std=0.02):
    w = synth.normal_bf16(seed, 0, V * H, std)
    hidden = synth.readout_hidden(seed, n, H)
    targets = synth.readout_targets(seed, n, V)
    return w, hidden, targets


@pytest.mark.parametrize("V,H,n", [(1000, 256, 300), (517, 64, 129), (256, 128, 128), (4099, 1024, 257)])
def test_margin_small_shapes_bf16(gpu, oracle, V, H, n):
    w, hidden, targets = problem(V, H, n)
    weight = gpu.upload_raw(w, BF16)
    margin, amax, tl = diagnosis.readout_margin(gpu, weight, None, V, H, hidden, targets)
    ref = oracle.readout_rows(w, oracle.BF16, None, V, H, synth.bf16_to_f32(hidden), targets)
    check_rows(margin, amax, tl, ref, 1e-5)


def test_margin_f32_hidden_and_bias(gpu, oracle):
    V, H, n = 3001, 512, 200
    w, _, targets = problem(V, H, n)
    hidden = synth.normal_f32(5, 9, n * H).reshape(n, H)
    bias = synth.normal_f32(5, 10, V, 0.5)
    weight = gpu.upload_raw(w, BF16)
    margin, amax, tl = diagnosis.readout_margin(gpu, weight, gpu.upload_f32(bias), V, H, hidden, targets)
    ref = oracle.readout_rows(w, oracle.BF16, bias, V, H, hidden, targets)
    check_rows(margin, amax, tl, ref, 1e-5)


@pytest.mark.parametrize("kind", ["plane", "joint"])
def test_margin_with_edits(gpu, oracle, kind):
    V, H, n = 2053, 256, 160
    w, hidden, targets = problem(V, H, n)
    h32 = synth.bf16_to_f32(hidden)
    if kind == "plane":
        rng = np.random.default_rng(1)
        u = rng.standard_normal(H)
        u /= np.linalg.norm(u)
        v = rng.standard_normal(H)
        v -= (v @ u) * u
        v /= np.linalg.norm(v)
        spec = ReadoutRotation(u, v, 0.35)
    else:
        spec = lsx.random_subspace_rotation(H, 16, 3.0, seed=4)
    edited = np.stack([spec.apply(h) for h in h32.astype(np.float64)]).astype(np.float32)
    ref = oracle.readout_rows(w, oracle.BF16, None, V, H, edited, targets)
    weight = gpu.upload_raw(w, BF16)
    rot = DeviceRotation.upload_edit(gpu, spec, H)
    for h in (hidden, h32):  # bf16 rows, and the same rows as f32 (hi/lo planes)
        margin, amax, tl = diagnosis.readout_margin(gpu, weight, None, V, H, h, targets, rot)
        check_rows(margin, amax, tl, ref, 1e-5)


@pytest.mark.parametrize("rank", [5, 70, 130])
def test_margin_with_wide_edits(gpu, oracle, rank):
    """Edit ranks that are not multiples of 8, and ranks that need more than one
    pass of the edit-image kernel (64 ranks per pass)."""
    V, H, n = 1031, 256, 96
    w, hidden, targets = problem(V, H, n)
    h32 = synth.bf16_to_f32(hidden)
    spec = lsx.random_subspace_rotation(H, rank, 3.0, seed=6)
    edited = np.stack([spec.apply(h) for h in h32.astype(np.float64)]).astype(np.float32)
    ref = oracle.readout_rows(w, oracle.BF16, None, V, H, edited, targets)
    weight = gpu.upload_raw(w, BF16)
    rot = DeviceRotation.upload_edit(gpu, spec, H)
    margin, amax, tl = diagnosis.readout_margin(gpu, weight, None, V, H, hidden, targets, rot)
    check_rows(margin, amax, tl, ref, 1e-5)


def test_ties_resolve_to_lowest_index(gpu, oracle):
    """Duplicate vocab rows produce exact ties: first argmax, lowest-index competitor."""
    V, H, n = 600, 64, 130
    w, hidden, _ = problem(V, H, n)
    w = w.reshape(V, H)
    w[300:600] = w[0:300]  # rows j and j + 300 give equal logits
    w = w.reshape(-1)
    ref_in = synth.bf16_to_f32(hidden)
    targets = np.zeros(n, np.uint32)
    for i in range(n):
        z = oracle.matvec(w, oracle.BF16, ref_in[i], None, V, H)
        targets[i] = int(np.argsort(z)[-3]) % 300 + (300 if i % 2 else 0)
    weight = gpu.upload_raw(w, BF16)
    margin, amax, tl = diagnosis.readout_margin(gpu, weight, None, V, H, hidden, targets)
    m_ref, a_ref, t_ref = oracle.readout_rows(w, oracle.BF16, None, V, H, ref_in, targets)
    assert np.array_equal(amax, a_ref)
    assert np.all(amax < 300)
    assert np.allclose(margin, m_ref, atol=1e-6)


def test_rejects_bad_arguments(gpu):
    weight = gpu.upload_raw(synth.normal_bf16(1, 0, 100 * 64), BF16)
    with pytest.raises(lsx.LsxError):
        diagnosis.readout_margin(gpu, weight, None, 100, 64, np.zeros((2, 64), np.float32), np.array([0, 100]))
    with pytest.raises(lsx.LsxError):
        diagnosis.readout_margin(gpu, weight, None, 101, 64, np.zeros((2, 64), np.float32), np.array([0, 1]))


def test_readout_validation_workload_full_size(gpu, oracle):
    """4096 RMSNorm'd bf16 hidden states x lm_head [151936, 1024] bf16 with a rank-16
    Givens edit (angles within 3 degrees); rows sampled for the oracle."""
    V, H, n = 151936, 1024, 4096
    w, hidden, targets = problem(V, H, n, seed=7)
    spec = lsx.random_subspace_rotation(H, 16, 3.0, seed=7)
    weight = gpu.upload_raw(w, BF16)
    rot = DeviceRotation.upload_edit(gpu, spec, H)
    margin, amax, tl = diagnosis.readout_margin(gpu, weight, None, V, H, hidden, targets, rot)
    sample = np.arange(0, n, 97)
    h = synth.bf16_to_f32(hidden[sample]).astype(np.float64)
    edited = np.stack([spec.apply(x) for x in h]).astype(np.float32)
    ref = oracle.readout_rows(w, oracle.BF16, None, V, H, edited, targets[sample])
    check_rows(margin[sample], amax[sample], tl[sample], ref, 1e-5)


def test_verify_cached_on_tiny_model(gpu, oracle, golden_tiny):
    """verify_cached: target prefixes through the fused kernel, protected prefixes
    through Model::readout; acceptance as src/diagnosis.rs:562-563."""
    model = lsx.Model.load(GOLDEN / "tiny_qwen3", gpu, 32)
    tokens, _, frames = model.generate(golden_tiny["prompt"], 6, frames=True)
    path_t = diagnosis.ObservedPath(0, False, [int(t) for t in tokens], frames)
    path_p = diagnosis.ObservedPath(1, True, [int(t) for t in tokens], frames)
    spec = lsx.random_subspace_rotation(model.hidden_size, 4, 0.01, seed=2)
    v = diagnosis.verify_cached(model, gpu, [int(tokens[-1])], spec, [path_t, path_p], margin=-100.0,
                                tolerance=1.0, deadline=diagnosis.Deadline.after(60))
    assert v.requested_answers_generated and v.protected_sequences_preserved and v.accepted
    ref = oracle.OracleModel(GOLDEN / "tiny_qwen3", 32)
    margins = [oracle.minimum_margin(ref.readout(f.hidden, spec.apply), int(t)) for f, t in zip(frames, tokens)]
    assert abs(v.target_min_margin - min(margins)) < 1e-4
    assert v.readout_calls == 2 * len(frames)


def test_compact_readout_matches_oracle(gpu, oracle):
    """CompactReadout (src/diagnosis.rs:608-666): z = z0 + F ((R - I) x) per
    observation, checked against the oracle's f32 matvec with the baseline as bias
    (the linear tolerance of tests/gpu.rs:19-40), and its deadline and finiteness
    checks."""
    V, r, n = 4099, 16, 5
    rng = np.random.default_rng(11)
    images = [rng.standard_normal(V).astype(np.float32) * 0.1 for _ in range(r)]
    baseline = [rng.standard_normal(V).astype(np.float32) for _ in range(n)]
    coordinates = [rng.standard_normal(r) for _ in range(n)]
    q, _ = np.linalg.qr(rng.standard_normal((r, r)))
    compact = diagnosis.CompactReadout(gpu, images, baseline, coordinates)
    got = compact.evaluate(gpu, q, diagnosis.Deadline(60.0))
    F = np.stack(images, axis=1)  # [V, r]
    delta = (q - np.eye(r)) @ np.stack(coordinates, axis=1)
    for i in range(n):
        want = oracle.matvec(F, 0, delta[:, i].astype(np.float32), baseline[i], V, r)
        assert np.all(np.abs(got[i] - want) <= 2e-6 * (1 + np.abs(want)))
    with pytest.raises(diagnosis.BudgetExpired):
        compact.evaluate(gpu, q, diagnosis.Deadline(0.0))
    bad = [b.copy() for b in baseline]
    bad[2][7] = np.inf
    with pytest.raises(ValueError):
        diagnosis.CompactReadout(gpu, images, bad, coordinates).evaluate(gpu, q, diagnosis.Deadline(60.0))


def test_host_entry_large_upload_matches_device_entry(gpu):
    """Host rows above the staging threshold (10.6 MB of f32, three pieces, the
    last one partial) give the same margins as the device-pointer entry."""
    import ctypes as C

    import torch

    from laplacesscissors_b200._lib import F32, check, lib
    V, H, n = 4099, 1024, 2600
    w, _, targets = problem(V, H, n)
    hidden = synth.normal_f32(8, 1, n * H).reshape(n, H)
    weight = gpu.upload_raw(w, BF16)
    margin, amax, tl = diagnosis.readout_margin(gpu, weight, None, V, H, hidden, targets)
    dev = torch.device("cuda", gpu.device)
    h = torch.from_numpy(hidden).to(dev)
    t = torch.from_numpy(targets.astype(np.uint32).view(np.int32)).to(dev)
    ws = torch.empty(lib.lsx_readout_workspace_bytes(V, H, n, None), dtype=torch.uint8, device=dev)
    out = torch.empty(n * 16, dtype=torch.uint8, device=dev)
    torch.cuda.synchronize(dev)
    base = out.data_ptr()
    check(lib.lsx_readout_margin_device(gpu.handle, weight.handle, None, V, H, C.c_void_p(h.data_ptr()), F32, n,
                                        C.c_void_p(t.data_ptr()), None, C.c_void_p(base), C.c_void_p(base + n * 8),
                                        C.c_void_p(base + n * 12), C.c_void_p(ws.data_ptr()), ws.numel()))
    gpu.synchronize()
    raw = out.cpu().numpy()
    assert np.array_equal(margin, raw[: n * 8].view(np.float64))
    assert np.array_equal(amax, raw[n * 8: n * 12].view(np.uint32))
    assert np.array_equal(tl, raw[n * 12:].view(np.float32))


def test_device_entries_report_status(gpu):
    """The device-pointer entries leave the kernels' status in the caller's
    workspace: lsx_readout_status reports non-finite scores (the reference's
    rejection, src/model.rs:680-683) for lsx_readout_margin_device and
    lsx_readout_shard_device, and a clean status after a clean call on the same
    workspace."""
    import ctypes as C

    import torch

    from laplacesscissors_b200._lib import F32, LsxError, check, lib
    V, H, n = 1031, 256, 48
    dev = f"cuda:{gpu.device}"
    weight = gpu.upload_raw(synth.normal_bf16(6, 0, V * H, 0.02), BF16)
    clean = synth.normal_f32(6, 9, n * H)
    bad = clean.copy()
    bad[7 * H + 3] = np.inf
    targets = torch.from_numpy(synth.readout_targets(6, n, V).astype(np.int32)).to(dev)
    ws_bytes = lib.lsx_readout_workspace_bytes(V, H, n, None)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    margin = torch.empty(n, dtype=torch.float64, device=dev)
    amax = torch.empty(n, dtype=torch.int32, device=dev)
    keys = torch.empty(n, dtype=torch.int64, device=dev)
    tlog = torch.empty(n, dtype=torch.float32, device=dev)
    for rows in (bad, clean):
        hidden = torch.from_numpy(rows).to(dev)
        check(lib.lsx_readout_margin_device(gpu.handle, weight.handle, None, V, H, C.c_void_p(hidden.data_ptr()), F32,
                                            n, C.c_void_p(targets.data_ptr()), None, C.c_void_p(margin.data_ptr()),
                                            C.c_void_p(amax.data_ptr()), None, C.c_void_p(ws.data_ptr()), ws_bytes))
        if rows is bad:
            with pytest.raises(LsxError) as err:
                check(lib.lsx_readout_status(gpu.handle, C.c_void_p(ws.data_ptr())))
            assert err.value.status == 4
        else:
            check(lib.lsx_readout_status(gpu.handle, C.c_void_p(ws.data_ptr())))
        check(lib.lsx_readout_shard_device(gpu.handle, weight.handle, None, 0, V, H, C.c_void_p(hidden.data_ptr()),
                                           F32, n, C.c_void_p(targets.data_ptr()), None, C.c_void_p(keys.data_ptr()),
                                           C.c_void_p(tlog.data_ptr()), C.c_void_p(ws.data_ptr()), ws_bytes))
        if rows is bad:
            with pytest.raises(LsxError) as err:
                check(lib.lsx_readout_status(gpu.handle, C.c_void_p(ws.data_ptr())))
            assert err.value.status == 4
        else:
            check(lib.lsx_readout_status(gpu.handle, C.c_void_p(ws.data_ptr())))
