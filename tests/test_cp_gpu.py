"""Context-parallel prefill on one GPU: every rank of a W-rank zigzag schedule
is run in turn in this process, with the all-gather replaced by handing each
rank the whole key/value sequence directly. The partial attention and the
log-sum-exp merge are the CUDA library's (g4a_prefill with position offsets,
g4a_lse_merge); the result must match the oracle's causal prefill of the whole
sequence.

Tolerance: max |diff| <= 2e-3 (bf16 inputs, as the single-launch prefill).
"""
import sys
from pathlib import Path

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


@pytest.mark.parametrize("world,T", [(2, 512), (4, 512), (8, 1024)])
def test_cp_prefill_matches_oracle(oracle, ctx, torch_cuda, world, T):
    from g4attn import cp
    torch = torch_cuda
    hd = 512
    r = rng(4000 + world)
    q = oracle.round_bf16(unit_rms_rows(r.standard_normal((T, 8, hd)).astype(np.float32)))
    k = oracle.round_bf16(unit_rms_rows(r.standard_normal((T, hd)).astype(np.float32)))
    v = oracle.round_bf16(r.standard_normal((T, hd)).astype(np.float32))
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda().to(torch.bfloat16)
    chunks = [cp.zigzag_chunks(T, world, rank) for rank in range(world)]
    keys, values = dev(k), dev(v)
    attend = cp.g4a_attend(ctx, torch, hd)
    merge = cp.g4a_merge(ctx, torch, hd)
    got = np.full((T, 8, hd), np.nan, np.float32)
    for rank in range(world):
        qc = [dev(q[a:b]) for a, b in chunks[rank]]
        kc = [dev(k[a:b]) for a, b in chunks[rank]]
        vc = [dev(v[a:b]) for a, b in chunks[rank]]
        gather = lambda kc, vc: ((lambda: None), keys, values)
        outs = cp.cp_prefill(qc, kc, vc, T, world, rank, gather, attend, merge)
        ctx.sync()
        for (a, b), o in zip(chunks[rank], outs):
            got[a:b] = o.cpu().numpy()
    want = oracle.prefill_attend(q, k, v, 8, 0)
    assert max_abs_diff(got, want) <= TOL


@pytest.mark.parametrize("world,T", [(2, 512), (4, 1024)])
def test_kv_shard_merge_matches_oracle(oracle, ctx, torch_cuda, world, T):
    """The key/value-shard partition's arithmetic on one GPU: each emulated
    rank's partial outputs and log-sum-exps over all rows (g4a_prefill on its
    two key chunks, g4a_lse_merge of the two), then the cross-rank maximum,
    weights and sums that the all-reduce and reduce-scatter carry, done here
    in one process; every rank's rows match the oracle's causal prefill."""
    from g4attn import cp
    torch = torch_cuda
    hd = 512
    r = rng(5000 + world)
    q = oracle.round_bf16(unit_rms_rows(r.standard_normal((T, 8, hd)).astype(np.float32)))
    k = oracle.round_bf16(unit_rms_rows(r.standard_normal((T, hd)).astype(np.float32)))
    v = oracle.round_bf16(r.standard_normal((T, hd)).astype(np.float32))
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda().to(torch.bfloat16)
    be = cp.TorchKvShardBackend(ctx, torch, None, hd)
    q_all = dev(q)
    rows = cp.rank_rows(T, world)
    parts = []
    for rank in range(world):
        chunks = cp.zigzag_chunks(T, world, rank)
        probs = cp.kv_shard_problems(T, world, rank)
        res = be.attend(probs, q_all, [dev(k[a:b]) for a, b in chunks], [dev(v[a:b]) for a, b in chunks])
        parts.append(be.partial(T, probs, res))
    m = torch.stack([p[1] for p in parts]).amax(0)
    x = sum(be.to_rank_order(be.scale(o, be.weights(l, m)), rows) for o, l in parts)
    w = sum(be.to_rank_order(be.weights(l, m), rows) for o, l in parts)
    got = be.finish(x, w)
    ctx.sync()
    ref = oracle.prefill_attend(q, k, v, 8, 0)
    want = np.concatenate([ref[a:b] for a, b in rows])
    assert max_abs_diff(got.cpu().numpy(), want) <= TOL


@pytest.fixture(scope="module")
def comm1(torch_cuda):
    """A one-rank NCCL communicator made by the library (g4a_nccl_*)."""
    import g4attn
    c = g4attn.NcclComm(1, 0, g4attn.nccl_unique_id(), 0)
    yield c
    c.close()


@pytest.mark.parametrize("schedule", ["kv_shards", "gather_kv"])
@pytest.mark.parametrize("hd,T", [(512, 1024), (256, 640)])
def test_cp_prefill_c_entry_one_rank(oracle, ctx, comm1, torch_cuda, schedule, hd, T):
    """g4a_cp_prefill through the C ABI on a one-rank communicator: both
    schedules run their whole path (NCCL gathers, all-reduce and
    reduce-scatter over one rank, the local and exchanged phases, the merges)
    and give the causal prefill of the whole sequence, against the oracle;
    per-phase device times are recorded; g4a_cp_wait returns OK."""
    import g4attn
    torch = torch_cuda
    sched = g4attn.CP_KV_SHARDS if schedule == "kv_shards" else g4attn.CP_GATHER_KV
    r = rng(6000 + hd + T)
    q = oracle.round_bf16(unit_rms_rows(r.standard_normal((T, 8, hd)).astype(np.float32)))
    k = oracle.round_bf16(unit_rms_rows(r.standard_normal((T, hd)).astype(np.float32)))
    v = oracle.round_bf16(r.standard_normal((T, hd)).astype(np.float32))
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda().to(torch.bfloat16)
    out = torch.full((T, 8, hd), float("nan"), device="cuda")
    ctx.profile(True)
    for _ in range(2):  # the second call reuses the context's exchange buffers and prepared lists
        ctx.cp_prefill(comm1.ptr, sched, hd, T, dev(q), dev(k), dev(v), out)
    ctx.cp_wait(comm1.ptr, 60000)
    phases = {name: ctx.profile_read(kid) for name, kid in
              (("exchange", g4attn.K_CP_EXCHANGE), ("local", g4attn.K_CP_ATTEND_LOCAL),
               ("remote", g4attn.K_CP_ATTEND_REMOTE), ("merge", g4attn.K_CP_MERGE))}
    ctx.profile(False)
    assert all(n > 0 for _, n in phases.values()), phases
    want = oracle.prefill_attend(q, k, v, 8, 0)
    assert max_abs_diff(out.cpu().numpy(), want) <= TOL


def test_cp_prefill_rejects_bad_calls(ctx, comm1, torch_cuda):
    import g4attn
    torch = torch_cuda
    x = torch.zeros(64, 8, 512, device="cuda", dtype=torch.bfloat16)
    kv = torch.zeros(64, 512, device="cuda", dtype=torch.bfloat16)
    out = torch.empty(64, 8, 512, device="cuda")
    for args in ((g4attn.CP_KV_SHARDS, 512, 63), (g4attn.CP_GATHER_KV, 128, 64), (7, 512, 64)):
        with pytest.raises(g4attn.EngError) as e:
            ctx.cp_prefill(comm1.ptr, args[0], args[1], args[2], x, kv, kv, out)
        assert e.value.code == g4attn.COMPUTE
    with pytest.raises(g4attn.EngError) as e:
        ctx.cp_prefill(0, g4attn.CP_KV_SHARDS, 512, 64, x, kv, kv, out)
    assert e.value.code == g4attn.COMPUTE
