"""Failure handling on the GPU, in the form that faults and hangs nothing: a
kernel's bounded wait is made to run out (g4a_debug_stall: the next launch
waits about 2 ms on a device word that nothing sets, records the time-out and
skips its work). The call then reports G4A_TIMEOUT -- the reference reports
failures as EngError results (crates/llm-eng/src/error.rs:3-15) -- and the
context stays usable: the next call is clean and matches the oracle.
"""
import numpy as np
import pytest

from helpers import max_abs_diff, norm_weight, normal, rng, unit_rms_rows

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _step_args(torch, oracle, hp, r, layers, w):
    args, raw = [], {}
    for layer in layers:
        hd = oracle.head_dim(hp, layer)
        q, k, v = normal(r, 8 * hd), normal(r, hd), normal(r, hd)
        raw[layer] = (q, k, v)
        args.append(dict(layer=layer, q_raw=torch.from_numpy(q).cuda(), k_raw=torch.from_numpy(k).cuda(),
                         v_raw=torch.from_numpy(v).cuda(), q_norm_w=torch.from_numpy(w[layer][0]).cuda(),
                         k_norm_w=torch.from_numpy(w[layer][1]).cuda(), out=torch.empty(8 * hd, device="cuda")))
    return args, raw


def test_decode_wait_timeout_then_clean_steps(oracle, torch_cuda):
    """The f16 paged decode's main kernel times out: g4a_sync returns
    G4A_TIMEOUT once; the step's appends (done by the prep kernel) stay, as
    the oracle's step does; the next step through g4a_decode and a
    host-buffer step through g4a_decode_host (which reports its own time-out
    directly) then match the oracle."""
    import g4attn
    torch = torch_cuda
    hp = oracle.hparams_e2b()
    ff = oracle.proportional_rope_freq_factors(512, 0.25)
    r = rng(99)
    ctx = g4attn.Context(0, max_positions=512)
    kv = g4attn.KvCache(ctx, 1, 512, dtype=g4attn.KV_F16, layers=[13, 14])
    okv = oracle.KvCache()
    w = {l: (norm_weight(r, oracle.head_dim(hp, l)), norm_weight(r, oracle.head_dim(hp, l))) for l in (13, 14)}
    hist = 150
    for layer in (13, 14):
        hd = oracle.head_dim(hp, layer)
        glob = oracle.layer_is_global(hp, layer)
        base = hp.global_rope_base if glob else hp.local_rope_base
        k_raw, v_raw = normal(r, hist, hd), normal(r, hist, hd)
        kv.append_tokens(0, layer, torch.from_numpy(k_raw).cuda(), torch.from_numpy(v_raw).cuda(),
                         torch.from_numpy(w[layer][1]).cuda())
        for t in range(hist):
            k = oracle.rope_neox(oracle.rms_norm(k_raw[t], w[layer][1]), t, base, hd, ff if glob else None)
            okv.append(layer, oracle.round_f16(k), oracle.round_f16(oracle.rms_norm(v_raw[t], None)))

    def oracle_step(pos, raw):
        return [okv.attention_block(hp, layer, pos, *raw[layer], w[layer][0], w[layer][1], ff, kv_store=1)
                for layer in (13, 14)]

    # 1. stalled step
    args, raw = _step_args(torch, oracle, hp, r, (13, 14), w)
    ctx.debug_stall(g4attn.K_DECODE_MAIN)
    ctx.decode(kv, args, [0], [hist])
    with pytest.raises(g4attn.EngError) as e:
        ctx.sync()
    assert e.value.code == g4attn.TIMEOUT
    oracle_step(hist, raw)
    ctx.sync()  # the flag was cleared
    # 2. clean device-pointer step
    args, raw = _step_args(torch, oracle, hp, r, (13, 14), w)
    ctx.decode(kv, args, [0], [hist + 1])
    ctx.sync()
    for a, want in zip(args, oracle_step(hist + 1, raw)):
        assert max_abs_diff(a["out"].cpu().numpy(), want) <= 1e-4
    # 3. host-buffer steps: a stalled one reports G4A_TIMEOUT itself, then a clean one
    for stalled, pos in ((True, hist + 2), (False, hist + 3)):
        host, raw = [], {}
        for layer in (13, 14):
            hd = oracle.head_dim(hp, layer)
            q, k, v = normal(r, 8 * hd), normal(r, hd), normal(r, hd)
            raw[layer] = (q, k, v)
            host.append(dict(layer=layer, q_raw=q, k_raw=k, v_raw=v, q_norm_w=torch.from_numpy(w[layer][0]).cuda(),
                             k_norm_w=torch.from_numpy(w[layer][1]).cuda(), out=np.zeros(8 * hd, np.float32)))
        if stalled:
            ctx.debug_stall(g4attn.K_DECODE_MAIN)
            with pytest.raises(g4attn.EngError) as e:
                ctx.decode_host(kv, host, [0], [pos])
            assert e.value.code == g4attn.TIMEOUT
            oracle_step(pos, raw)
        else:
            ctx.decode_host(kv, host, [0], [pos])
            for h, want in zip(host, oracle_step(pos, raw)):
                assert max_abs_diff(h["out"], want) <= 1e-4
    kv.close()
    ctx.close()


def test_prefill_wait_timeout_then_clean_call(oracle, torch_cuda):
    """The tcgen05 prefill times out in every CTA pair (both widths in one
    launch): g4a_sync returns G4A_TIMEOUT; the same call again is clean and
    matches the oracle."""
    import g4attn
    torch = torch_cuda
    ctx = g4attn.Context(0)
    r = rng(98)
    probs, want = [], []
    for hd, window in ((256, 64), (512, 0)):
        T = 160
        q = oracle.round_bf16(unit_rms_rows(r.standard_normal((T, 8, hd)).astype(np.float32)))
        k = oracle.round_bf16(unit_rms_rows(r.standard_normal((T, hd)).astype(np.float32)))
        v = oracle.round_bf16(r.standard_normal((T, hd)).astype(np.float32))
        dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda().to(torch.bfloat16)
        probs.append(dict(head_dim=hd, window=window, n_q=T, n_kv=T, q=dev(q), k=dev(k), v=dev(v),
                          out=torch.full((T, 8, hd), float("nan"), device="cuda")))
        want.append(oracle.prefill_attend(q, k, v, 8, window))
    args = ctx.prefill_args(probs)
    ctx.debug_stall(g4attn.K_PREFILL)
    ctx.prefill(args)
    with pytest.raises(g4attn.EngError) as e:
        ctx.sync()
    assert e.value.code == g4attn.TIMEOUT
    ctx.prefill(args)
    ctx.sync()
    for p, w_ in zip(probs, want):
        assert max_abs_diff(p["out"].cpu().numpy(), w_) <= 2e-3
    ctx.close()


def test_debug_stall_only_for_kernels_with_a_stall_test(torch_cuda):
    import g4attn
    ctx = g4attn.Context(0)
    with pytest.raises(g4attn.EngError) as e:
        ctx.debug_stall(g4attn.K_MATVEC_Q8)
    assert e.value.code == g4attn.COMPUTE
    ctx.close()
