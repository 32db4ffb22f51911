"""Decode-path parity on the GPU: the CUDA library through its C ABI against
the CPU oracle on identical seeded inputs.

Tolerances: decode attention outputs within max |diff| <= 1e-4 (the f32
decode bar); the q/k norm + RoPE + append path is bit-exact.
"""
import numpy as np
import pytest

from helpers import max_abs_diff, norm_weight, normal, rng

pytestmark = pytest.mark.gpu

TOL = 1e-4


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


@pytest.fixture(scope="module")
def g4a():
    import g4attn
    return g4attn


@pytest.fixture(scope="module")
def ctx(g4a, torch_cuda):
    c = g4a.Context(0, max_positions=4200)
    yield c
    c.close()


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    return t.detach().cpu().numpy()


def processed_kv(oracle, hp, layer, k_raw, v_raw, kw, positions, ff):
    """k = rope(rms_norm(k_raw, kw)), v = rms_norm(v_raw) per row (model.rs:402-404)."""
    glob = oracle.layer_is_global(hp, layer)
    hd = k_raw.shape[1]
    base = hp.global_rope_base if glob else hp.local_rope_base
    ks, vs = [], []
    positions = list(positions)
    if not positions:
        return np.zeros((0, k_raw.shape[1]), np.float32), np.zeros((0, k_raw.shape[1]), np.float32)
    for row, pos in enumerate(positions):
        k = oracle.rms_norm(k_raw[row], kw, hp.rms_norm_eps)
        k = oracle.rope_neox(k, pos, base, hd, ff if glob else None)
        ks.append(k)
        vs.append(oracle.rms_norm(v_raw[row], None, hp.rms_norm_eps))
    return np.stack(ks).astype(np.float32), np.stack(vs).astype(np.float32)


@pytest.mark.parametrize("hd,length", [(256, 1), (256, 17), (256, 512), (512, 628), (512, 1), (256, 1000)])
def test_attend_matches_oracle(oracle, ctx, torch_cuda, hd, length):
    r = rng(hd + length)
    q = normal(r, 8 * hd) / np.float32(np.sqrt(hd))
    k, v = normal(r, length, hd), normal(r, length, hd)
    out = torch_cuda.empty(8 * hd, device="cuda")
    ctx.attend(dev(torch_cuda, q), dev(torch_cuda, k), dev(torch_cuda, v), 8, 1, 1.0, out)
    ctx.sync()
    want = oracle.attend(q, k, v, 8, 1)
    assert max_abs_diff(host(out), want) <= TOL


@pytest.mark.parametrize("n_heads,n_kv,hd,length", [(4, 2, 8, 5), (4, 2, 16, 9), (8, 8, 64, 33)])
def test_attend_generic_shapes(oracle, ctx, torch_cuda, n_heads, n_kv, hd, length):
    r = rng(n_heads * hd + length)
    q = normal(r, n_heads * hd)
    k, v = normal(r, length, n_kv * hd), normal(r, length, n_kv * hd)
    out = torch_cuda.empty(n_heads * hd, device="cuda")
    ctx.attend(dev(torch_cuda, q), dev(torch_cuda, k), dev(torch_cuda, v), n_heads, n_kv, 1.0, out)
    ctx.sync()
    assert max_abs_diff(host(out), oracle.attend(q, k, v, n_heads, n_kv)) <= TOL


def test_attend_scale_and_empty(g4a, oracle, ctx, torch_cuda):
    r = rng(4)
    q, k, v = normal(r, 8 * 256), normal(r, 40, 256), normal(r, 40, 256)
    out = torch_cuda.empty(8 * 256, device="cuda")
    ctx.attend(dev(torch_cuda, q), dev(torch_cuda, k), dev(torch_cuda, v), 8, 1, 0.0625, out)
    ctx.sync()
    assert max_abs_diff(host(out), oracle.attend(q, k, v, 8, 1, 0.0625)) <= TOL
    with pytest.raises(g4a.EngError) as e:
        ctx.attend(dev(torch_cuda, q), None, None, 8, 1, 1.0, out, length=0)
    assert e.value.code == g4a.NONFINITE


def test_attend_nonfinite_reported(g4a, ctx, torch_cuda):
    r = rng(5)
    q = normal(r, 8 * 256)
    q[3] = np.nan
    k, v = normal(r, 8, 256), normal(r, 8, 256)
    out = torch_cuda.empty(8 * 256, device="cuda")
    ctx.attend(dev(torch_cuda, q), dev(torch_cuda, k), dev(torch_cuda, v), 8, 1, 1.0, out)
    with pytest.raises(g4a.EngError) as e:
        ctx.sync()
    assert e.value.code == g4a.NONFINITE
    ctx.sync()  # the flag was cleared


@pytest.mark.parametrize("layer,dtype", [(13, 0), (14, 0), (13, 1), (14, 1)])
def test_append_tokens_bit_exact(g4a, oracle, ctx, torch_cuda, layer, dtype):
    """norm + RoPE + store through the device equals the oracle bit for bit
    (f32 storage) or its binary16 rounding (f16 storage)."""
    hp = oracle.hparams_e2b()
    hd = oracle.head_dim(hp, layer)
    ff = oracle.proportional_rope_freq_factors(512, 0.25)
    r = rng(layer * 7 + dtype)
    T = 130
    k_raw, v_raw, kw = normal(r, T, hd), normal(r, T, hd), norm_weight(r, hd)
    kv = g4a.KvCache(ctx, 2, 256, dtype=dtype, layers=[layer])
    kv.append_tokens(1, layer, dev(torch_cuda, k_raw), dev(torch_cuda, v_raw), dev(torch_cuda, kw))
    assert kv.len(1, layer) == T and kv.len(0, layer) == 0
    ko = torch_cuda.empty(T, hd, device="cuda")
    vo = torch_cuda.empty(T, hd, device="cuda")
    kv.view(1, layer, T, ko, vo)
    ctx.sync()
    k_ref, v_ref = processed_kv(oracle, hp, layer, k_raw, v_raw, kw, range(T), ff)
    if dtype == 1:
        k_ref, v_ref = oracle.round_f16(k_ref), oracle.round_f16(v_ref)
    assert np.array_equal(host(ko), k_ref)
    assert np.array_equal(host(vo), v_ref)
    kv.close()


def test_kv_view_errors(g4a, ctx, torch_cuda):
    """context_memory.rs:53-69 / :109-116 through the device cache."""
    kv = g4a.KvCache(ctx, 1, 128, layers=[13])
    o = torch_cuda.empty(4, 256, device="cuda")
    with pytest.raises(g4a.EngError) as e:
        kv.view(0, 14, 1, o, o)
    assert e.value.code == g4a.MISSING_LAYER
    kv.view(0, 14, 0, o, o)  # a missing layer is fine for len 0
    with pytest.raises(g4a.EngError) as e:
        kv.view(0, 13, 1, o, o)
    assert e.value.code == g4a.CONTEXT_TOO_LONG
    rows = torch_cuda.ones(2, 256, device="cuda")
    kv.append(0, 13, rows, rows)
    kv.view(0, 13, 2, o[:2], o[2:])
    with pytest.raises(g4a.EngError) as e:
        kv.view(0, 13, 3, o, o)
    assert e.value.code == g4a.CONTEXT_TOO_LONG
    kv.clear()
    assert kv.len(0, 13) == 0
    with pytest.raises(g4a.EngError) as e:
        kv.append(0, 14, rows, rows)
    assert e.value.code == g4a.MISSING_LAYER
    kv.close()


def _fill_history(g4a, oracle, torch, kv, okv, hp, seq, layer, n, r, kw, ff):
    """Appends n already-seen tokens to both caches (device: fused raw path;
    oracle: rows processed by the oracle)."""
    hd = oracle.head_dim(hp, layer)
    k_raw, v_raw = normal(r, n, hd), normal(r, n, hd)
    if n:
        kv.append_tokens(seq, layer, dev(torch, k_raw), dev(torch, v_raw), dev(torch, kw))
    k_ref, v_ref = processed_kv(oracle, hp, layer, k_raw, v_raw, kw, range(n), ff)
    if kv.dtype == 1:
        k_ref, v_ref = oracle.round_f16(k_ref), oracle.round_f16(v_ref)
    for i in range(n):
        okv.append(layer, k_ref[i], v_ref[i])


@pytest.mark.parametrize("dtype", [0, 1])
def test_decode_config0(g4a, oracle, ctx, torch_cuda, dtype):
    """Config 0: one decode step at position 627 on a sliding layer (13) and a
    global layer (14), the new token appended by the fused kernel; then the
    KV-shared layers 33 and 34 read those caches."""
    torch = torch_cuda
    hp = oracle.hparams_e2b()
    ff = oracle.proportional_rope_freq_factors(512, 0.25)
    r = rng(627 + dtype)
    kv = g4a.KvCache(ctx, 1, 1024, dtype=dtype, layers=[13, 14])
    okv = oracle.KvCache()
    w = {}
    for layer in (13, 14, 33, 34):
        hd = oracle.head_dim(hp, layer)
        w[layer] = (norm_weight(r, hd), norm_weight(r, hd))
    for layer in (13, 14):
        _fill_history(g4a, oracle, torch, kv, okv, hp, 0, layer, 627, r, w[layer][1], ff)
    pos = 627
    args, refs = [], []
    for layer in (13, 14):
        hd = oracle.head_dim(hp, layer)
        q_raw, k_raw, v_raw = normal(r, 8 * hd), normal(r, hd), normal(r, hd)
        out = torch.empty(8 * hd, device="cuda")
        args.append(dict(layer=layer, q_raw=dev(torch, q_raw), k_raw=dev(torch, k_raw), v_raw=dev(torch, v_raw),
                         q_norm_w=dev(torch, w[layer][0]), k_norm_w=dev(torch, w[layer][1]), out=out))
        refs.append(okv.attention_block(hp, layer, pos, q_raw, k_raw, v_raw, w[layer][0], w[layer][1], ff,
                                        kv_store=dtype))
    ctx.decode(kv, args, [0], [pos])
    ctx.sync()
    for a, ref in zip(args, refs):
        assert max_abs_diff(host(a["out"]), ref) <= TOL
    for layer in (13, 14):  # the appended row is the oracle's, bit for bit
        hd = oracle.head_dim(hp, layer)
        assert kv.len(0, layer) == 628
        ko, vo = torch.empty(628, hd, device="cuda"), torch.empty(628, hd, device="cuda")
        kv.view(0, layer, 628, ko, vo)
        k_ref, v_ref = okv.view(layer, 628)
        assert np.array_equal(host(ko), k_ref) and np.array_equal(host(vo), v_ref)
    # shared layers 33 (local -> 13) and 34 (global -> 14) at the same position
    args, refs = [], []
    for layer in (33, 34):
        hd = oracle.head_dim(hp, layer)
        q_raw = normal(r, 8 * hd)
        out = torch.empty(8 * hd, device="cuda")
        args.append(dict(layer=layer, q_raw=dev(torch, q_raw), q_norm_w=dev(torch, w[layer][0]), out=out))
        refs.append(okv.attention_block(hp, layer, pos, q_raw, None, None, w[layer][0], None, ff))
    ctx.decode(kv, args, [0], [pos])
    ctx.sync()
    for a, ref in zip(args, refs):
        assert max_abs_diff(host(a["out"]), ref) <= TOL
    assert kv.len(0, 13) == 628  # shared layers append nothing
    kv.close()


@pytest.mark.parametrize("dtype", [0, 1])
def test_decode_batched_paged(g4a, oracle, ctx, torch_cuda, dtype):
    """Config 2 shape at small scale: sequences at ragged lengths (page and
    window boundaries, length 1) decoded together on a local and a global
    layer in one call."""
    torch = torch_cuda
    hp = oracle.hparams_e2b()
    ff = oracle.proportional_rope_freq_factors(512, 0.25)
    lengths = [0, 62, 63, 64, 65, 510, 511, 512, 513, 700, 128, 1]
    n = len(lengths)
    r = rng(99 + dtype)
    kv = g4a.KvCache(ctx, n + 2, 1024, dtype=dtype, layers=[13, 14])
    okvs = [oracle.KvCache() for _ in range(n)]
    w = {l: (norm_weight(r, oracle.head_dim(hp, l)), norm_weight(r, oracle.head_dim(hp, l))) for l in (13, 14)}
    seq_ids = [s + 2 for s in range(n)]  # exercise a non-zero block-table row
    for s, L in enumerate(lengths):
        for layer in (13, 14):
            _fill_history(g4a, oracle, torch, kv, okvs[s], hp, seq_ids[s], layer, L, r, w[layer][1], ff)
    args, refs = [], {13: [], 14: []}
    raws = {}
    for layer in (13, 14):
        hd = oracle.head_dim(hp, layer)
        q_raw, k_raw, v_raw = normal(r, n, 8 * hd), normal(r, n, hd), normal(r, n, hd)
        raws[layer] = (q_raw, k_raw, v_raw)
        args.append(dict(layer=layer, q_raw=dev(torch, q_raw), k_raw=dev(torch, k_raw), v_raw=dev(torch, v_raw),
                         q_norm_w=dev(torch, w[layer][0]), k_norm_w=dev(torch, w[layer][1]),
                         out=torch.empty(n, 8 * hd, device="cuda")))
    ctx.decode(kv, args, seq_ids, lengths)
    ctx.sync()
    for a in args:
        layer = a["layer"]
        q_raw, k_raw, v_raw = raws[layer]
        got = host(a["out"])
        for s, L in enumerate(lengths):
            ref = okvs[s].attention_block(hp, layer, L, q_raw[s], k_raw[s], v_raw[s], w[layer][0], w[layer][1], ff,
                                          kv_store=dtype)
            assert max_abs_diff(got[s], ref) <= TOL, (layer, L)
    kv.close()


@pytest.mark.parametrize("dtype", [0, 1])
def test_decode_host_buffers(g4a, oracle, ctx, torch_cuda, dtype):
    """g4a_decode_host (q/k/v/out in page-locked host memory, one call per
    step): the outputs are g4a_decode's bit for bit on a cache with the same
    history, and the oracle's within the f32 decode bar; a KV-shared layer
    takes no k/v; a rejected call copies nothing and leaves the lengths; a
    non-finite score is reported by the call itself."""
    torch = torch_cuda
    hp = oracle.hparams_e2b()
    ff = oracle.proportional_rope_freq_factors(512, 0.25)
    lengths = [0, 63, 64, 511, 512, 700, 1]
    n = len(lengths)
    caches = []
    for _ in range(2):
        r = rng(321 + dtype)
        kv = g4a.KvCache(ctx, n, 1024, dtype=dtype, layers=[13, 14])
        okvs = [oracle.KvCache() for _ in range(n)]
        w = {l: (norm_weight(r, oracle.head_dim(hp, l)), norm_weight(r, oracle.head_dim(hp, l))) for l in (13, 14)}
        for s, L in enumerate(lengths):
            for layer in (13, 14):
                _fill_history(g4a, oracle, torch, kv, okvs[s], hp, s, layer, L, r, w[layer][1], ff)
        caches.append((kv, okvs))
    r = rng(400 + dtype)
    raws, dev_args, host_args = {}, [], []
    for layer in (13, 14):
        hd = oracle.head_dim(hp, layer)
        q_raw, k_raw, v_raw = normal(r, n, 8 * hd), normal(r, n, hd), normal(r, n, hd)
        raws[layer] = (q_raw, k_raw, v_raw)
        wq, wk = dev(torch, w[layer][0]), dev(torch, w[layer][1])
        dev_args.append(dict(layer=layer, q_raw=dev(torch, q_raw), k_raw=dev(torch, k_raw), v_raw=dev(torch, v_raw),
                             q_norm_w=wq, k_norm_w=wk, out=torch.empty(n, 8 * hd, device="cuda")))
        pin = lambda a: torch.from_numpy(np.ascontiguousarray(a)).pin_memory()
        host_args.append(dict(layer=layer, q_raw=pin(q_raw), k_raw=pin(k_raw), v_raw=pin(v_raw), q_norm_w=wq,
                              k_norm_w=wk, out=torch.full((n, 8 * hd), float("nan")).pin_memory()))
    seqs = list(range(n))
    ctx.decode(caches[0][0], dev_args, seqs, lengths)
    ctx.sync()
    args = g4a.DecodeHostArgs(host_args)
    ctx.decode_host(caches[1][0], args, seqs, lengths)
    for a, h in zip(dev_args, host_args):
        layer = a["layer"]
        got = h["out"].numpy()
        assert np.array_equal(got, host(a["out"])), layer
        q_raw, k_raw, v_raw = raws[layer]
        for s, L in enumerate(lengths):
            ref = caches[1][1][s].attention_block(hp, layer, L, q_raw[s], k_raw[s], v_raw[s], w[layer][0],
                                                  w[layer][1], ff, kv_store=dtype)
            assert max_abs_diff(got[s], ref) <= TOL, (layer, L)
    kv = caches[1][0]
    # a KV-shared layer (33 reads 13) from host buffers, no k/v
    q33 = normal(r, n, 8 * 256)
    out33 = np.full((n, 8 * 256), np.nan, np.float32)
    ctx.decode_host(kv, [dict(layer=33, q_raw=q33, q_norm_w=dev_args[0]["q_norm_w"], out=out33)], seqs,
                    [L for L in lengths])
    ctx.decode(caches[0][0], [dict(layer=33, q_raw=dev(torch, q33), q_norm_w=dev_args[0]["q_norm_w"],
                                   out=dev_args[0]["out"])], seqs, [L for L in lengths])
    ctx.sync()
    assert np.array_equal(out33, host(dev_args[0]["out"]))
    # rejected: position past the cache (view of more rows than held)
    before = [kv.len(s, 13) for s in seqs]
    out_bad = np.full((1, 8 * 256), 7.0, np.float32)
    with pytest.raises(g4a.EngError) as e:
        ctx.decode_host(kv, [dict(layer=13, q_raw=q33[:1].copy(), k_raw=raws[13][1][:1].copy(),
                                  v_raw=raws[13][2][:1].copy(), q_norm_w=dev_args[0]["q_norm_w"],
                                  k_norm_w=dev_args[0]["k_norm_w"], out=out_bad)], [0], [lengths[0] + 5])
    assert e.value.code == g4a.CONTEXT_TOO_LONG
    assert np.all(out_bad == 7.0) and [kv.len(s, 13) for s in seqs] == before
    # non-finite q: the call itself raises
    bad = q33[:1].copy()
    bad[:] = np.inf
    with pytest.raises(g4a.EngError) as e:
        ctx.decode_host(kv, [dict(layer=33, q_raw=bad, q_norm_w=dev_args[0]["q_norm_w"], out=out_bad)], [1],
                        [lengths[1]])
    assert e.value.code == g4a.NONFINITE
    for kv_, _ in caches:
        kv_.close()


def test_decode_errors(g4a, oracle, ctx, torch_cuda):
    torch = torch_cuda
    kv = g4a.KvCache(ctx, 2, 64, layers=[13])
    q = torch.zeros(8 * 256, device="cuda")
    k = torch.zeros(256, device="cuda")
    w = torch.ones(256, device="cuda")
    out = torch.empty(8 * 256, device="cuda")
    a = dict(layer=13, q_raw=q, k_raw=k, v_raw=k, q_norm_w=w, k_norm_w=w, out=out)
    with pytest.raises(g4a.EngError) as e:  # position 1 with an empty cache: view(2) of 1 row
        ctx.decode(kv, [a], [0], [1])
    assert e.value.code == g4a.CONTEXT_TOO_LONG
    with pytest.raises(g4a.EngError) as e:
        ctx.decode(kv, [dict(a, q_norm_w=None)], [0], [0])
    assert e.value.code == g4a.MISSING_WEIGHT
    with pytest.raises(g4a.EngError) as e:  # layer 14 is not held
        ctx.decode(kv, [dict(a, layer=14, q_raw=torch.zeros(8 * 512, device="cuda"),
                             out=torch.empty(8 * 512, device="cuda"))], [0], [0])
    assert e.value.code == g4a.MISSING_LAYER
    with pytest.raises(g4a.EngError) as e:  # shared layer 33 reads 13, which has no rows yet
        ctx.decode(kv, [dict(layer=33, q_raw=q, q_norm_w=w, out=out)], [0], [0])
    assert e.value.code == g4a.CONTEXT_TOO_LONG
    with pytest.raises(g4a.EngError) as e:
        ctx.decode(kv, [dict(a, layer=35)], [0], [0])
    assert e.value.code == g4a.BAD_LAYER
    with pytest.raises(g4a.EngError) as e:
        ctx.decode(kv, [a], [0, 0], [0, 0])
    assert e.value.code == g4a.COMPUTE
    with pytest.raises(g4a.EngError) as e:  # a shared layer together with its source
        ctx.decode(kv, [a, dict(layer=33, q_raw=q, q_norm_w=w, out=out)], [0], [0])
    assert e.value.code == g4a.COMPUTE
    for pos in range(64):  # fill to capacity, then one more is ContextTooLong
        ctx.decode(kv, [a], [1], [pos])
    with pytest.raises(g4a.EngError) as e:
        ctx.decode(kv, [a], [1], [64])
    assert e.value.code == g4a.CONTEXT_TOO_LONG
    ctx.sync()
    kv.close()


def test_decode_position_zero_and_nonfinite(g4a, oracle, ctx, torch_cuda):
    torch = torch_cuda
    hp = oracle.hparams_e2b()
    ff = oracle.proportional_rope_freq_factors(512, 0.25)
    r = rng(0)
    kv = g4a.KvCache(ctx, 1, 64, layers=[14])
    okv = oracle.KvCache()
    wq, wk = norm_weight(r, 512), norm_weight(r, 512)
    q_raw, k_raw, v_raw = normal(r, 8 * 512), normal(r, 512), normal(r, 512)
    out = torch.empty(8 * 512, device="cuda")
    a = dict(layer=14, q_raw=dev(torch, q_raw), k_raw=dev(torch, k_raw), v_raw=dev(torch, v_raw),
             q_norm_w=dev(torch, wq), k_norm_w=dev(torch, wk), out=out)
    ctx.decode(kv, [a], [0], [0])
    ctx.sync()
    ref = okv.attention_block(hp, 14, 0, q_raw, k_raw, v_raw, wq, wk, ff)
    assert max_abs_diff(host(out), ref) <= TOL
    bad = q_raw.copy()
    bad[:] = np.inf
    ctx.decode(kv, [dict(a, q_raw=dev(torch, bad))], [0], [1])
    with pytest.raises(g4a.EngError) as e:
        ctx.sync()
    assert e.value.code == g4a.NONFINITE
    kv.close()


def test_plan_runs_match_decode(g4a, oracle, ctx, torch_cuda):
    """A staged plan gives the oracle's result, on every repeated run."""
    torch = torch_cuda
    hp = oracle.hparams_e2b()
    ff = oracle.proportional_rope_freq_factors(512, 0.25)
    r = rng(77)
    lengths = [5, 300, 900]
    kv = g4a.KvCache(ctx, 3, 1024, dtype=1, layers=[14])
    okvs = [oracle.KvCache() for _ in lengths]
    wq, wk = norm_weight(r, 512), norm_weight(r, 512)
    for s, L in enumerate(lengths):
        _fill_history(g4a, oracle, torch, kv, okvs[s], hp, s, 14, L, r, wk, ff)
    q_raw, k_raw, v_raw = normal(r, 3, 8 * 512), normal(r, 3, 512), normal(r, 3, 512)
    out = torch.empty(3, 8 * 512, device="cuda")
    a = dict(layer=14, q_raw=dev(torch, q_raw), k_raw=dev(torch, k_raw), v_raw=dev(torch, v_raw),
             q_norm_w=dev(torch, wq), k_norm_w=dev(torch, wk), out=out)
    plan = ctx.decode_plan(kv, [a], [0, 1, 2], lengths)
    assert kv.len(1, 14) == 301
    refs = [okvs[s].attention_block(hp, 14, L, q_raw[s], k_raw[s], v_raw[s], wq, wk, ff, kv_store=1)
            for s, L in enumerate(lengths)]
    first = None
    for _ in range(3):
        out.fill_(float("nan"))
        plan.run()
        ctx.sync()
        got = host(out)
        for s in range(3):
            assert max_abs_diff(got[s], refs[s]) <= TOL
        if first is None:
            first = got.copy()
        assert np.array_equal(got, first)  # deterministic combine order
    plan.close()
    kv.close()


def test_decode_both_widths_long_contexts(g4a, oracle, ctx, torch_cuda):
    """Both layer kinds in one call at long contexts: tasks split across many
    items, items of both head widths interleaved on the same CTAs, combined
    by the merge kernel; two consecutive steps."""
    torch = torch_cuda
    hp = oracle.hparams_e2b()
    ff = oracle.proportional_rope_freq_factors(512, 0.25)
    r = rng(4242)
    lengths = [4000, 3100, 2600, 1999, 1500, 1024, 777, 513, 300, 64, 33, 2]
    n = len(lengths)
    kv = g4a.KvCache(ctx, n, 4100, dtype=1, layers=[13, 14])
    okvs = [oracle.KvCache() for _ in range(n)]
    w = {l: (norm_weight(r, oracle.head_dim(hp, l)), norm_weight(r, oracle.head_dim(hp, l))) for l in (13, 14)}
    for s, L in enumerate(lengths):
        for layer in (13, 14):
            _fill_history(g4a, oracle, torch, kv, okvs[s], hp, s, layer, L, r, w[layer][1], ff)
    for step in range(2):
        args, raws = [], {}
        for layer in (13, 14):
            hd = oracle.head_dim(hp, layer)
            q_raw, k_raw, v_raw = normal(r, n, 8 * hd), normal(r, n, hd), normal(r, n, hd)
            raws[layer] = (q_raw, k_raw, v_raw)
            args.append(dict(layer=layer, q_raw=dev(torch, q_raw), k_raw=dev(torch, k_raw),
                             v_raw=dev(torch, v_raw), q_norm_w=dev(torch, w[layer][0]),
                             k_norm_w=dev(torch, w[layer][1]), out=torch.empty(n, 8 * hd, device="cuda")))
        pos = [L + step for L in lengths]
        ctx.decode(kv, args, list(range(n)), pos)
        ctx.sync()
        for a in args:
            layer = a["layer"]
            q_raw, k_raw, v_raw = raws[layer]
            got = host(a["out"])
            for s in range(n):
                ref = okvs[s].attention_block(hp, layer, pos[s], q_raw[s], k_raw[s], v_raw[s], w[layer][0],
                                              w[layer][1], ff, kv_store=1)
                assert max_abs_diff(got[s], ref) <= TOL, (step, layer, lengths[s])
    kv.close()


def test_decode_host_in_place_small_step(g4a, oracle, ctx, torch_cuda):
    """A small host-buffer step (one sequence, both layers: 55 KB) with every
    buffer page-locked runs in place (the kernels read q/k/v and write the
    output over the bus): bit for bit g4a_decode's on a twin cache, and the
    oracle's within the decode bar; a second step in a row as well."""
    torch = torch_cuda
    hp = oracle.hparams_e2b()
    ff = oracle.proportional_rope_freq_factors(512, 0.25)
    r = rng(555)
    L = 300
    caches = []
    for _ in range(2):
        rr = rng(556)
        kv = g4a.KvCache(ctx, 1, 512, dtype=1, layers=[13, 14])
        okv = oracle.KvCache()
        w = {l: (norm_weight(rr, oracle.head_dim(hp, l)), norm_weight(rr, oracle.head_dim(hp, l))) for l in (13, 14)}
        for layer in (13, 14):
            _fill_history(g4a, oracle, torch, kv, okv, hp, 0, layer, L, rr, w[layer][1], ff)
        caches.append((kv, okv))
    pin = lambda a: torch.from_numpy(np.ascontiguousarray(a)).pin_memory()
    for step in range(2):
        dev_args, host_args, raws = [], [], {}
        for layer in (13, 14):
            hd = oracle.head_dim(hp, layer)
            q_raw, k_raw, v_raw = normal(r, 1, 8 * hd), normal(r, 1, hd), normal(r, 1, hd)
            raws[layer] = (q_raw, k_raw, v_raw)
            wq, wk = dev(torch, w[layer][0]), dev(torch, w[layer][1])
            dev_args.append(dict(layer=layer, q_raw=dev(torch, q_raw), k_raw=dev(torch, k_raw),
                                 v_raw=dev(torch, v_raw), q_norm_w=wq, k_norm_w=wk,
                                 out=torch.empty(1, 8 * hd, device="cuda")))
            host_args.append(dict(layer=layer, q_raw=pin(q_raw), k_raw=pin(k_raw), v_raw=pin(v_raw), q_norm_w=wq,
                                  k_norm_w=wk, out=torch.full((1, 8 * hd), float("nan")).pin_memory()))
        ctx.decode(caches[0][0], dev_args, [0], [L + step])
        ctx.sync()
        ctx.decode_host(caches[1][0], host_args, [0], [L + step])
        for a, h in zip(dev_args, host_args):
            layer = a["layer"]
            got = h["out"].numpy()
            assert np.array_equal(got, host(a["out"])), (step, layer)
            ref = caches[1][1].attention_block(hp, layer, L + step, *raws[layer], w[layer][0], w[layer][1], ff,
                                               kv_store=1)
            assert max_abs_diff(got[0], ref) <= TOL, (step, layer)
    for kv_, _ in caches:
        kv_.close()
