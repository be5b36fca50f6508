"""Q4_0 vecmat (ComputeBackend::q4_vecmat, backend.rs:56-60) and the batched gate+up pair
(ComputeBackend::q4_matvec_pair_batch, backend.rs:64-69) on the GPU vs the CPU oracle.

References: crates/larql-compute/csrc/q4_dot.c:201-232 (q4_0_vecmat_c: per row scale = f16(d) * act, rows with
-1e-10 < act < 1e-10 skipped); crates/larql-compute/src/metal/ops/q4_batched.rs:19-80 (per position
quantize_to_q8, then the Q4_0 x Q8 matvec of q4_dot.c:169-199 on gate and up).
Tolerance: max |err| <= 1e-3 * ||y_ref||_inf.
"""
import os

import numpy as np
import pytest

import oracle as O
from conftest import max_err_ok, normal, seed_for

pytestmark = pytest.mark.gpu
L = pytest.importorskip("larql_cuda")
torch = pytest.importorskip("torch")

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "q4_0_ref.npz")


def _cmp(got, ref, what):
    ok, err, bound = max_err_ok(got, ref)
    assert ok, f"{what}: max err {err} > {bound}"


def test_vecmat_golden_from_reference_kernel(backend):
    """The reference's own q4_0_vecmat_c output (8 x 64, its test shape) from the committed fixture."""
    g = np.load(GOLDEN)
    inter, hidden = int(g["x86_vecmat.rows"]), int(g["x86_vecmat.hidden"])
    got = backend.q4_vecmat(g["x86_vecmat.x"], g["x86_vecmat.q4"], inter, hidden)
    _cmp(got, g["x86_vecmat.y"], "golden vecmat")


# hidden 992 = 31 blocks (one partial column group), 4128 = 129 blocks (a last group of one block),
# 32 = a single block; 14336 x 4096 is the FFN down projection the reference's walk path uses it for.
@pytest.mark.parametrize("inter,hidden", [(64, 32), (300, 992), (1000, 4128), (10240, 2560), (14336, 4096),
                                          (7, 1024)])
def test_vecmat_vs_oracle(backend, inter, hidden):
    w = O.quantize_q4_0(normal(seed_for("vm", inter, hidden), inter * hidden, 0.02))
    act = normal(seed_for("vma", inter, hidden), inter)
    got = backend.q4_vecmat(act, w, inter, hidden)
    _cmp(got, O.q4_0_vecmat(act, w, inter, hidden), f"vecmat {inter}x{hidden}")


def test_vecmat_zero_skip_semantics(backend):
    """Rows whose activation lies strictly inside (-1e-10, 1e-10) are never read: a NaN scale there stays out
    of the output; the same row with a live activation makes every column of its blocks NaN; a NaN
    activation is not skipped."""
    inter, hidden = 96, 512
    w = O.quantize_q4_0(normal(3, inter * hidden, 0.02)).reshape(inter, hidden // 32, 18).copy()
    w[10, :, 0:2] = np.frombuffer(np.uint16(0x7E00).tobytes(), np.uint8)  # NaN f16 scale in every block
    act = normal(4, inter)
    act[::5] = np.float32(5e-11)
    act[10] = np.float32(-9.9e-11)
    act[11] = np.float32(1e-10)   # boundary: not skipped
    got = backend.q4_vecmat(act, w.reshape(-1), inter, hidden)
    ref = O.q4_0_vecmat(act, w.reshape(-1), inter, hidden)
    assert np.all(np.isfinite(ref)) and np.all(np.isfinite(got))
    _cmp(got, ref, "skipped NaN row")
    act[10] = np.float32(0.5)
    got = backend.q4_vecmat(act, w.reshape(-1), inter, hidden)
    assert np.all(np.isnan(got)) and np.all(np.isnan(O.q4_0_vecmat(act, w.reshape(-1), inter, hidden)))
    act[10] = np.float32(-9.9e-11)
    act[50] = np.nan
    got = backend.q4_vecmat(act, w.reshape(-1), inter, hidden)
    assert np.all(np.isnan(got))


def test_vecmat_zero_activation_and_device_form(backend):
    inter, hidden = 4096, 2048
    w = O.quantize_q4_0(normal(5, inter * hidden, 0.02))
    assert np.all(backend.q4_vecmat(np.zeros(inter, np.float32), w, inter, hidden) == 0.0)
    wt = backend.register_weight(w, L.FMT_Q4_0, inter, hidden)
    act = normal(6, inter)
    ad = torch.from_numpy(act).cuda()
    out = torch.full((hidden,), float("nan"), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    backend.q4_vecmat_dev(wt, ad, out)
    backend.sync()
    got = out.cpu().numpy()
    backend.q4_vecmat_dev(wt, ad, out)
    backend.sync()
    wt.release()
    assert np.array_equal(got.view(np.uint32), out.cpu().numpy().view(np.uint32))
    _cmp(got, O.q4_0_vecmat(act, w, inter, hidden), "device vecmat")


def _pair_ref(wg, wu, x, rows, hidden):
    gs, us = [], []
    for t in range(x.shape[0]):
        q8, s8 = O.quantize_to_q8(x[t])
        gs.append(O.q4_0_matvec_q8(wg, q8, s8, rows, hidden))
        us.append(O.q4_0_matvec_q8(wu, q8, s8, rows, hidden))
    return np.stack(gs), np.stack(us)


@pytest.mark.parametrize("seq,rows,hidden", [(1, 300, 1024), (6, 1000, 2560), (3, 14336, 4096)])
def test_pair_batch_vs_oracle(backend, seq, rows, hidden):
    wg = O.quantize_q4_0(normal(seed_for("pbg", rows, hidden), rows * hidden, 0.02))
    wu = O.quantize_q4_0(normal(seed_for("pbu", rows, hidden), rows * hidden, 0.02))
    x = normal(seed_for("pbx", seq, hidden), seq * hidden).reshape(seq, hidden)
    g, u = backend.q4_matvec_pair_batch(wg, wu, x, seq, rows, hidden)
    rg, ru = _pair_ref(wg, wu, x, rows, hidden)
    for t in range(seq):
        _cmp(g[t], rg[t], f"gate t{t}")
        _cmp(u[t], ru[t], f"up t{t}")


def test_pair_batch_device_form_and_shape_check(backend):
    seq, rows, hidden = 4, 512, 1024
    wg = O.quantize_q4_0(normal(7, rows * hidden, 0.02))
    wu = O.quantize_q4_0(normal(8, rows * hidden, 0.02))
    tg = backend.register_weight(wg, L.FMT_Q4_0, rows, hidden)
    tu = backend.register_weight(wu, L.FMT_Q4_0, rows, hidden)
    x = normal(9, seq * hidden).reshape(seq, hidden)
    xd = torch.from_numpy(x).cuda()
    go = torch.empty(seq * rows, dtype=torch.float32, device="cuda")
    uo = torch.empty(seq * rows, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    backend.q4_matvec_pair_batch_dev(tg, tu, xd, seq, go, uo)
    backend.sync()
    rg, ru = _pair_ref(wg, wu, x, rows, hidden)
    _cmp(go.cpu().numpy().reshape(seq, rows), rg, "device gate")
    _cmp(uo.cpu().numpy().reshape(seq, rows), ru, "device up")
    tw = backend.register_weight(O.quantize_q4_0(normal(10, 256 * hidden, 0.02)), L.FMT_Q4_0, 256, hidden)
    with pytest.raises(L.LarqlCudaError):
        backend.q4_matvec_pair_batch_dev(tg, tw, xd, seq, go, uo)
    for t_ in (tg, tu, tw):
        t_.release()


def _random_q4_0_blocks(seed, rows, hidden):
    """Random Q4_0 bytes whose f16 scales include subnormals (q4_dot.c decodes them exactly)."""
    from conftest import random_f16_bits
    rng = np.random.default_rng(seed)
    nb = rows * hidden // 32
    b = rng.integers(0, 256, size=(nb, 18), dtype=np.uint8)
    d = random_f16_bits(rng, nb, -12, 1)
    d[::3] = rng.integers(1, 0x3FF, d[::3].size).astype(np.uint16)
    b[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
    return b.reshape(-1)


def test_pair_batch_many_positions_random_blocks(backend):
    """19 positions (weight passes of 8, 8 and 3 positions on the tensor-core form) over random-byte Q4_0 blocks with
    subnormal scales."""
    seq, rows, hidden = 19, 700, 2048
    wg = _random_q4_0_blocks(51, rows, hidden)
    wu = _random_q4_0_blocks(52, rows, hidden)
    x = normal(53, seq * hidden).reshape(seq, hidden)
    g, u = backend.q4_matvec_pair_batch(wg, wu, x, seq, rows, hidden)
    rg, ru = _pair_ref(wg, wu, x, rows, hidden)
    for t in range(seq):
        _cmp(g[t], rg[t], f"gate t{t}")
        _cmp(u[t], ru[t], f"up t{t}")
