"""Q8_0 mat-vec family on the GPU through the C ABI against the oracle's
restatement of crates/llm-backend-cpu/src/matvec.rs.

Bars: everything is bit-exact: the quantized activations, the plain mat-vec
(integer block dot products, block values summed in block order from -0.0,
as the reference), and GEGLU and soft-cap, whose tanh is the device
restatement of glibc's tanhf (the reference's f32::tanh on Linux).
"""
import numpy as np
import pytest

from helpers import rng

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


@pytest.fixture(scope="module")
def ctx(torch_cuda):
    import g4attn
    c = g4attn.Context(0)
    yield c
    c.close()


def weights(oracle, seed, rows, cols, scale=0.05):
    return oracle.q8_0_bytes_of(rng(seed).standard_normal(rows * cols).astype(np.float32) * scale)


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def oracle_rows(oracle, fn, w, rows, cols, x, *extra):
    outs = []
    for v in range(x.shape[0]):
        s, q = oracle.quantize_q8_0(x[v])
        outs.append(fn(*w, rows, cols, s, q, *extra))
    return np.stack(outs)


def test_quantize_bit_exact(oracle, ctx, torch_cuda):
    torch = torch_cuda
    x = rng(1).standard_normal(4096).astype(np.float32) * 3
    x[:32] = 0.0                      # zero block: scale 0, quants 0
    x[32:64] = 0.0
    x[32], x[33], x[34] = 127.0, 2.5, -3.5  # the reference's known answer
    scales = torch.empty(128, device="cuda")
    quants = torch.empty(4096, dtype=torch.int8, device="cuda")
    ctx.quantize_q8_0(dev(torch, x), 4096, scales, quants)
    ctx.sync()
    ws, wq = oracle.quantize_q8_0(x)
    assert np.array_equal(scales.cpu().numpy(), ws)
    assert np.array_equal(quants.cpu().numpy(), wq)
    assert ws[1] == 1.0 and wq[32:36].tolist() == [127, 2, -4, 0]


@pytest.mark.parametrize("rows,cols,n_vec", [
    (64, 256, 1),      # the reference test's shape
    (1031, 1536, 1),   # E2B width (d_model), rows not a multiple of the tile
    (300, 6144, 3),    # wide rows, several vectors in one pass
    (257, 512, 9),     # more vectors than one pass holds
    (33, 96, 2),       # cols not a multiple of 256: the generic kernel
    (0, 256, 1),       # no rows
    (1000, 1536, 100), # many vectors: the tensor-core kernel, ragged row and vector tiles
    (64, 256, 64),     # one stage of K, whole tiles
    (200, 3072, 17),   # d_ff-wide rows
])
def test_matvec_bit_exact(oracle, ctx, torch_cuda, rows, cols, n_vec):
    torch = torch_cuda
    w = weights(oracle, rows + cols, rows, cols)
    x = rng(cols + n_vec).standard_normal((n_vec, cols)).astype(np.float32)
    out = torch.full((n_vec, rows), float("nan"), device="cuda")
    ctx.matvec_q8_0(dev(torch, w), rows, cols, dev(torch, x), out, n_vec=n_vec)
    ctx.sync()
    want = oracle_rows(oracle, oracle.matvec_q8_0, (w,), rows, cols, x)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32).reshape(n_vec, rows))


def test_matvec_reference_fixtures(oracle, ctx, torch_cuda):
    """The reference test's own inputs (LCG values, its weight quantizer)."""
    torch = torch_cuda
    rows, cols = 64, 256
    w = oracle.q8_0_bytes_of(oracle.lcg_values(1, rows * cols))
    x = oracle.lcg_values(2, cols)[None, :]
    out = torch.empty(1, rows, device="cuda")
    ctx.matvec_q8_0(dev(torch, w), rows, cols, dev(torch, x), out)
    ctx.sync()
    assert np.array_equal(out.cpu().numpy(), oracle_rows(oracle, oracle.matvec_q8_0, (w,), rows, cols, x))


def test_matvec_unaligned_weights(oracle, ctx, torch_cuda):
    """Weights that start 2 bytes into a buffer (a GGUF tensor at an even
    offset) take the generic kernel and give the same bits."""
    torch = torch_cuda
    rows, cols = 100, 512
    w = weights(oracle, 5, rows, cols)
    buf = torch.zeros(len(w) + 16, dtype=torch.uint8, device="cuda")
    buf[2:2 + len(w)] = dev(torch, w)
    x = rng(6).standard_normal((1, cols)).astype(np.float32)
    out = torch.empty(1, rows, device="cuda")
    ctx.matvec_q8_0(buf[2:], rows, cols, dev(torch, x), out)
    ctx.sync()
    assert np.array_equal(out.cpu().numpy(), oracle_rows(oracle, oracle.matvec_q8_0, (w,), rows, cols, x))


def close(got, want):
    return np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("rows,cols,n_vec", [(300, 256, 1), (1000, 1536, 2), (50, 96, 1), (333, 1536, 70)])
def test_geglu(oracle, ctx, torch_cuda, rows, cols, n_vec):
    torch = torch_cuda
    gate, up = weights(oracle, 7, rows, cols), weights(oracle, 8, rows, cols)
    x = rng(9).standard_normal((n_vec, cols)).astype(np.float32)
    out = torch.empty(n_vec, rows, device="cuda")
    ctx.geglu_q8_0(dev(torch, gate), dev(torch, up), rows, cols, dev(torch, x), out, n_vec=n_vec)
    ctx.sync()
    assert close(out.cpu().numpy(), oracle_rows(oracle, oracle.geglu_q8_0, (gate, up), rows, cols, x))


def test_softcap_logits(oracle, ctx, torch_cuda):
    """The output head's form: soft-cap 30 over the mat-vec (model.rs:438-449)."""
    torch = torch_cuda
    rows, cols = 4099, 1536
    w = weights(oracle, 10, rows, cols, scale=0.5)
    x = rng(11).standard_normal((1, cols)).astype(np.float32)
    out = torch.empty(1, rows, device="cuda")
    ctx.matvec_q8_0_softcap(dev(torch, w), rows, cols, dev(torch, x), 30.0, out)
    ctx.sync()
    assert close(out.cpu().numpy(), oracle_rows(oracle, oracle.matvec_q8_0_softcap, (w,), rows, cols, x, 30.0))


def test_softcap_logits_batched(oracle, ctx, torch_cuda):
    """The head over many sequences at once (the batched decoder's form)."""
    torch = torch_cuda
    rows, cols, n_vec = 777, 1536, 40
    w = weights(oracle, 12, rows, cols, scale=0.5)
    x = rng(13).standard_normal((n_vec, cols)).astype(np.float32)
    out = torch.empty(n_vec, rows, device="cuda")
    ctx.matvec_q8_0_softcap(dev(torch, w), rows, cols, dev(torch, x), 30.0, out, n_vec=n_vec)
    ctx.sync()
    assert close(out.cpu().numpy(), oracle_rows(oracle, oracle.matvec_q8_0_softcap, (w,), rows, cols, x, 30.0))


def test_shape_errors(ctx, torch_cuda):
    import g4attn
    torch = torch_cuda
    x = torch.zeros(1, 100, device="cuda")
    out = torch.empty(1, 4, device="cuda")
    w = torch.zeros(1000, dtype=torch.uint8, device="cuda")
    with pytest.raises(g4attn.EngError) as e:
        ctx.matvec_q8_0(w, 4, 100, x, out)
    assert e.value.code == g4attn.COMPUTE and "multiple of 32" in e.value.message
