"""Prefill parity on the GPU: the tcgen05 kernel through the C ABI against the
oracle's token-at-a-time attention (the reference's prompt loop) on the same
bf16-rounded inputs.

Tolerance: max |diff| <= 2e-3 (bf16 inputs, f32 accumulation, fp16 P).
"""
import numpy as np
import pytest

from helpers import max_abs_diff, rng, unit_rms_rows

pytestmark = pytest.mark.gpu

TOL = 2e-3


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


def make_qkv(oracle, seed, n_q, n_kv, hd):
    """Unit-RMS Q (per head) and K rows, N(0,1) V, rounded to bf16."""
    r = rng(seed)
    q = unit_rms_rows(r.standard_normal((n_q, 8, hd)).astype(np.float32))
    k = unit_rms_rows(r.standard_normal((n_kv, hd)).astype(np.float32))
    v = r.standard_normal((n_kv, hd)).astype(np.float32)
    return oracle.round_bf16(q), oracle.round_bf16(k), oracle.round_bf16(v)


def to_dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda().to(torch.bfloat16)


def reference(q, k, v, window, q_pos0=0, kv_pos0=0):
    """float64 statement of the per-position attention with absolute
    positions (eng/mod.rs:10-36 per query position) plus the log-sum-exp."""
    n_q, H, hd = q.shape
    n_kv = k.shape[0]
    qpos = q_pos0 + np.arange(n_q)
    kpos = kv_pos0 + np.arange(n_kv)
    s = np.einsum("thd,kd->thk", q.astype(np.float64), k.astype(np.float64))
    vis = (kpos[None, :] <= qpos[:, None])
    if window:
        vis &= (qpos[:, None] - kpos[None, :]) < window
    s = np.where(vis[:, None, :], s, -np.inf)
    m = s.max(-1, keepdims=True)
    has = np.isfinite(m)
    e = np.where(has, np.exp(s - np.where(has, m, 0)), 0.0)
    l = e.sum(-1, keepdims=True)
    out = np.where(has, (e @ v.astype(np.float64)) / np.where(has, l, 1), 0.0)
    lse = np.where(has[..., 0], (m + np.log(np.where(has, l, 1)))[..., 0], -np.inf)
    return out, lse


def run(ctx, torch, q, k, v, hd, window, q_pos0=0, kv_pos0=0, lse=False):
    n_q, n_kv = q.shape[0], k.shape[0]
    out = torch.full((n_q, 8, hd), float("nan"), device="cuda")
    lse_t = torch.full((n_q, 8), float("nan"), device="cuda") if lse else None
    ctx.prefill([dict(head_dim=hd, window=window, n_q=n_q, q_pos0=q_pos0, n_kv=n_kv, kv_pos0=kv_pos0,
                      q=to_dev(torch, q), k=to_dev(torch, k), v=to_dev(torch, v), out=out, lse=lse_t)])
    ctx.sync()
    return out.cpu().numpy(), (lse_t.cpu().numpy() if lse else None)


@pytest.mark.parametrize("hd,T,window", [(256, 1, 512), (256, 17, 512), (256, 200, 64), (512, 200, 0),
                                          (512, 130, 0), (256, 628, 512)])
def test_prefill_matches_oracle(oracle, ctx, torch_cuda, hd, T, window):
    q, k, v = make_qkv(oracle, hd * 1000 + T, T, T, hd)
    got, _ = run(ctx, torch_cuda, q, k, v, hd, window)
    want = oracle.prefill_attend(q, k, v, 8, window)
    assert max_abs_diff(got, want) <= TOL


def test_prefill_global_628(oracle, ctx, torch_cuda):
    """Config 1's global layer shape: 628 tokens, 512-wide heads, full causal."""
    q, k, v = make_qkv(oracle, 628, 628, 628, 512)
    got, _ = run(ctx, torch_cuda, q, k, v, 512, 0)
    want = oracle.prefill_attend(q, k, v, 8, 0)
    assert max_abs_diff(got, want) <= TOL


@pytest.mark.parametrize("hd,window,n_q,q_pos0,n_kv,kv_pos0", [
    (512, 0, 100, 300, 400, 0),    # a chunk of queries against the whole prefix
    (512, 0, 64, 128, 128, 256),   # keys all in the future: no visible key
    (256, 512, 90, 700, 300, 500), # window crossing the key block start
    (512, 0, 40, 1000, 200, 900),  # keys of a later shard only partly visible
])
def test_prefill_offsets_and_lse(oracle, ctx, torch_cuda, hd, window, n_q, q_pos0, n_kv, kv_pos0):
    q, k, v = make_qkv(oracle, n_q + n_kv, n_q, n_kv, hd)
    got, lse = run(ctx, torch_cuda, q, k, v, hd, window, q_pos0, kv_pos0, lse=True)
    want, want_lse = reference(q, k, v, window, q_pos0, kv_pos0)
    assert max_abs_diff(got, want) <= TOL
    fin = np.isfinite(want_lse)
    assert np.array_equal(np.isfinite(lse), fin)
    if fin.any():
        assert np.max(np.abs(lse[fin] - want_lse[fin])) <= 1e-3


def test_prefill_rescale_path(oracle, ctx, torch_cuda):
    """Scores that grow along the keys force the running max up by more than
    2^15 several times (the lazy O rescale); the result still matches."""
    hd, T = 256, 512
    q, k, v = make_qkv(oracle, 7, T, T, hd)
    ramp = np.linspace(0.2, 3.0, T, dtype=np.float32)[:, None]
    k = oracle.round_bf16(k * ramp)
    got, _ = run(ctx, torch_cuda, q, k, v, hd, 0)
    want = oracle.prefill_attend(q, k, v, 8, 0)
    assert max_abs_diff(got, want) <= TOL


def test_prefill_35_layers_one_launch(oracle, ctx, torch_cuda):
    """Config 1: all 35 layer-equivalents in one call, layers 15-34 reusing
    the K/V of layer 13 (local) or 14 (global). Each layer equals the same
    problem run alone, bit for bit, and two layers match the oracle."""
    import g4attn
    torch = torch_cuda
    hp = g4attn.hparams_e2b()
    T = 628
    kvs = {}
    probs, qs = [], []
    for layer in range(35):
        src, _ = g4attn.kv_source_layer(hp, layer)
        hd = g4attn.head_dim(hp, layer)
        glob = g4attn.layer_is_global(hp, layer)
        if src not in kvs:
            _, k, v = make_qkv(oracle, 500 + src, 1, T, hd)
            kvs[src] = (k, v, to_dev(torch, k), to_dev(torch, v))
        q, _, _ = make_qkv(oracle, 900 + layer, T, 1, hd)
        qs.append(q)
        probs.append(dict(head_dim=hd, window=0 if glob else 512, n_q=T, n_kv=T, q=to_dev(torch, q),
                          k=kvs[src][2], v=kvs[src][3], out=torch.empty(T, 8, hd, device="cuda")))
    ctx.prefill(probs)
    ctx.sync()
    for layer in (0, 14, 33, 34):
        p = probs[layer]
        alone = torch.empty_like(p["out"])
        ctx.prefill([dict(p, out=alone)])
        ctx.sync()
        assert torch.equal(alone, p["out"]), layer
    for layer in (13, 34):
        src, _ = g4attn.kv_source_layer(hp, layer)
        k, v = kvs[src][0], kvs[src][1]
        want = oracle.prefill_attend(qs[layer], k, v, 8, probs[layer]["window"])
        assert max_abs_diff(probs[layer]["out"].cpu().numpy(), want) <= TOL


def test_prefill_rejects_bad_shapes(ctx, torch_cuda):
    import g4attn
    torch = torch_cuda
    x = torch.zeros(16, 8, 128, device="cuda", dtype=torch.bfloat16)
    out = torch.empty(16, 8, 128, device="cuda")
    with pytest.raises(g4attn.EngError) as e:
        ctx.prefill([dict(head_dim=128, n_q=16, n_kv=16, q=x, k=x, v=x, out=out)])
    assert e.value.code == g4attn.COMPUTE


def test_prefill_shared_values_of_different_lengths(oracle, ctx, torch_cuda):
    """Problems that read one K/V pair over different key counts (the longer
    one listed second) and a problem with its own K/V, in one call: the fp16
    copy of a shared V covers the longest use, and every result matches."""
    torch = torch_cuda
    hd = 256
    q1, k, v = make_qkv(oracle, 11, 100, 300, hd)
    q2, _, _ = make_qkv(oracle, 12, 300, 1, hd)
    q3, k3, v3 = make_qkv(oracle, 13, 80, 80, 512)
    kd, vd = to_dev(torch, k), to_dev(torch, v)
    outs = [torch.full((n, 8, d), float("nan"), device="cuda") for n, d in ((100, hd), (300, hd), (80, 512))]
    ctx.prefill([
        dict(head_dim=hd, window=0, n_q=100, n_kv=100, q=to_dev(torch, q1), k=kd, v=vd, out=outs[0]),
        dict(head_dim=hd, window=64, n_q=300, n_kv=300, q=to_dev(torch, q2), k=kd, v=vd, out=outs[1]),
        dict(head_dim=512, window=0, n_q=80, n_kv=80, q=to_dev(torch, q3), k=to_dev(torch, k3), v=to_dev(torch, v3),
             out=outs[2]),
    ])
    ctx.sync()
    wants = [oracle.prefill_attend(q1, k[:100], v[:100], 8, 0), oracle.prefill_attend(q2, k, v, 8, 64),
             oracle.prefill_attend(q3, k3, v3, 8, 0)]
    for got, want in zip(outs, wants):
        assert max_abs_diff(got.cpu().numpy(), want) <= TOL


def test_prefill_repeated_list_reads_current_values(oracle, ctx, torch_cuda):
    """The library reuses its prepared launch for a repeated problem list;
    the inputs are still read afresh on every call (V changed in place between
    two identical calls is seen), and a different list afterwards is prepared
    anew."""
    torch = torch_cuda
    hd, T = 256, 150
    q, k, v = make_qkv(oracle, 21, T, T, hd)
    _, _, v2 = make_qkv(oracle, 22, 1, T, hd)
    qd, kd, vd = to_dev(torch, q), to_dev(torch, k), to_dev(torch, v)
    out = torch.empty(T, 8, hd, device="cuda")
    args = ctx.prefill_args([dict(head_dim=hd, window=0, n_q=T, n_kv=T, q=qd, k=kd, v=vd, out=out)])
    ctx.prefill(args)
    ctx.sync()
    assert max_abs_diff(out.cpu().numpy(), oracle.prefill_attend(q, k, v, 8, 0)) <= TOL
    vd.copy_(to_dev(torch, v2))
    ctx.prefill(args)
    ctx.sync()
    assert max_abs_diff(out.cpu().numpy(), oracle.prefill_attend(q, k, v2, 8, 0)) <= TOL
    out2 = torch.empty(T, 8, hd, device="cuda")
    ctx.prefill([dict(head_dim=hd, window=64, n_q=T, n_kv=T, q=qd, k=kd, v=vd, out=out2)])
    ctx.sync()
    assert max_abs_diff(out2.cpu().numpy(), oracle.prefill_attend(q, k, v2, 8, 64)) <= TOL


def sampled_rows(T, n, seed):
    """n query positions spread over [0, T): the first and last rows, rows on
    either side of 32-token row-tile and 128-key tile edges, and random rows."""
    edges = {0, 1, T - 1, T - 2}
    for e in (32, 128, 4096, T // 2):
        for m in (e, 2 * e, 3 * e, T - e):
            edges.update({m - 1, m})
    edges = sorted(x for x in edges if 0 <= x < T)
    r = rng(seed)
    rest = r.choice(np.setdiff1d(np.arange(T), edges), size=max(0, n - len(edges)), replace=False)
    return np.sort(np.concatenate([edges, rest]).astype(np.int64))


def test_prefill_config3_32768_sampled_rows(oracle, ctx, torch_cuda):
    """Configuration 3 at its benchmarked size: one 32,768-token global layer
    (512-wide heads, full causal) in one call, unit-RMS bf16 Q/K and N(0,1) V
    generated on the device. 256 query rows spread over the sequence (first,
    last, both sides of row-tile and key-tile edges, random) are checked
    against the oracle's attend over each row's causal keys [0, t] -- the
    reference's prompt loop at position t (model.rs:326-366 over
    eng/mod.rs:33-35's global range). This reaches what shorter cases do not:
    256 key tiles per item, TMA rows past 2^15, and the lazy rescale over 32k
    keys."""
    torch = torch_cuda
    T, hd = 32768, 512
    gen = torch.Generator(device="cuda")
    gen.manual_seed(32768)

    def unit(shape):
        x = torch.randn(*shape, device="cuda", generator=gen)
        return (x / x.pow(2).mean(-1, keepdim=True).sqrt()).to(torch.bfloat16)

    q, k = unit((T, 8, hd)), unit((T, hd))
    v = torch.randn(T, hd, device="cuda", generator=gen).to(torch.bfloat16)
    out = torch.full((T, 8, hd), float("nan"), device="cuda")
    ctx.prefill([dict(head_dim=hd, window=0, n_q=T, n_kv=T, q=q, k=k, v=v, out=out)])
    ctx.sync()
    rows = sampled_rows(T, 256, 3)
    assert len(rows) == 256
    idx = torch.from_numpy(rows).cuda()
    got = out.index_select(0, idx).cpu().numpy()
    q_h = q.index_select(0, idx).float().cpu().numpy()
    k_h, v_h = k.float().cpu().numpy(), v.float().cpu().numpy()
    del out
    oracle.pool_init(0)
    worst = 0.0
    for i, t in enumerate(rows):
        want = oracle.attend(q_h[i].reshape(-1), k_h[: t + 1], v_h[: t + 1], 8, 1, 1.0)
        worst = max(worst, max_abs_diff(got[i].reshape(-1), want))
    assert worst <= TOL, worst
