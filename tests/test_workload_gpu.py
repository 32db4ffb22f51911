"""Parity on the exact workload bench.py times for configuration 2: the 64
seeded contexts of one GPU (U[1, 4096]), the cache and step inputs built by
bench.build_decode with the bench's seed, one step run as the bench runs it
(a staged plan over layers 13 and 14). A stratified sample of 16 sequences
(every 4th by context length) is checked against the oracle's attention
block (model.rs:393-410 without the projections) fed the same raw rows,
at the f32 decode bar.
"""
import numpy as np
import pytest

from helpers import max_abs_diff

pytestmark = pytest.mark.gpu

TOL = 1e-4


def test_config2_bench_workload_sampled(oracle):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import bench
    import g4attn as g4a
    hp = oracle.hparams_e2b()
    ff = oracle.proportional_rope_freq_factors(512, 0.25)
    lengths = [int(c) for c in bench.shard(bench.global_lengths(1), 1, 0)]
    assert len(lengths) == bench.SEQS_PER_GPU
    order = np.argsort(lengths, kind="stable")
    sample = [int(s) for s in order[::4]]
    assert len(sample) == 16
    ctx = g4a.Context(0, max_positions=bench.MAX_CTX + 128)
    stream = torch.cuda.Stream()
    ctx.set_stream(stream.cuda_stream)
    kv, args, weights, kept = bench.build_decode(torch, g4a, ctx, lengths, 8, 1234, keep=set(sample))
    n = len(lengths)
    plan = ctx.decode_plan(kv, [args[bench.LOCAL_LAYER], args[bench.GLOBAL_LAYER]], list(range(n)),
                           [c - 1 for c in lengths])
    plan.run()
    ctx.sync()
    worst = 0.0
    for layer in (bench.LOCAL_LAYER, bench.GLOBAL_LAYER):
        a = args[layer]
        hd = oracle.head_dim(hp, layer)
        glob = oracle.layer_is_global(hp, layer)
        base = hp.global_rope_base if glob else hp.local_rope_base
        qn, kn = (w.cpu().numpy() for w in weights[layer])
        q_raw, k_raw, v_raw = (a[key].cpu().numpy() for key in ("q_raw", "k_raw", "v_raw"))
        got = a["out"].cpu().numpy()
        for s in sample:
            okv = oracle.KvCache()
            hist = lengths[s] - 1
            if hist:
                kh, vh = kept[(s, layer)]
                ks = np.stack([oracle.rope_neox(oracle.rms_norm(kh[t], kn, hp.rms_norm_eps), t, base, hd,
                                                ff if glob else None) for t in range(hist)])
                vs = np.stack([oracle.rms_norm(vh[t], None, hp.rms_norm_eps) for t in range(hist)])
                okv.append_rows(layer, oracle.round_f16(ks), oracle.round_f16(vs))
            want = okv.attention_block(hp, layer, hist, q_raw[s], k_raw[s], v_raw[s], qn, kn, ff, kv_store=1)
            d = max_abs_diff(got[s], want)
            worst = max(worst, d)
            assert d <= TOL, (layer, s, lengths[s], d)
    plan.close()
    kv.close()
    ctx.close()
    print(f"config 2 workload: 16 of 64 sequences, contexts {lengths[sample[0]]}..{lengths[sample[-1]]}, "
          f"max |diff| {worst:.3g}")
