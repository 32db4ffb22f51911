"""Context-parallel prefill schedules on CPU ranks (gloo, world size 2 and 4),
with a float64 numpy stand-in for the attention arithmetic; the result must
equal plain causal attention:
* the all-gather schedule: zigzag chunking, the key/value all-gather, which
  (query, key) chunk pairs each rank computes, the local log-sum-exp merge;
* the key/value-shard schedule: each rank's partials over all rows, the
  all-reduce of the maxima and the reduce-scatter of the weighted sums."""
import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]


def _np_attend(problems, q_chunks, keys_of, values_of):
    outs = []
    for p in problems:
        q = q_chunks[p.q_chunk].astype(np.float64)  # [n, 8, hd]
        k = keys_of(p).astype(np.float64)
        v = values_of(p).astype(np.float64)
        qpos = np.arange(p.q0, p.q1)[:, None, None]
        kpos = np.arange(p.k0, p.k1)[None, None, :]
        s = np.einsum("thd,kd->thk", q, k)
        s = np.where(kpos <= qpos, s, -np.inf)
        m = s.max(-1, keepdims=True)
        has = np.isfinite(m)
        e = np.where(has, np.exp(s - np.where(has, m, 0)), 0.0)
        l = e.sum(-1, keepdims=True)
        out = np.where(has, (e @ v) / np.where(has, l, 1), 0.0)
        lse = np.where(has[..., 0], (m + np.log(np.where(has, l, 1)))[..., 0], -np.inf)
        outs.append((out, lse))
    return outs


def _np_merge(parts):
    lse = np.stack([p[1] for p in parts])  # [P, n, 8]
    M = lse.max(0)
    w = np.where(np.isfinite(lse), np.exp(lse - np.where(np.isfinite(M), M, 0)), 0.0)
    L = w.sum(0)
    out = sum(w[i][..., None] * parts[i][0] for i in range(len(parts)))
    return out / np.where(L > 0, L, 1)[..., None]


def _rank_main(rank, world, port, T, hd, result_dir):
    sys.path.insert(0, str(ROOT / "gemma4-rs_b200"))
    import torch
    import torch.distributed as dist
    from g4attn import cp
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    r = np.random.default_rng(7)
    q = r.standard_normal((T, 8, hd)) / np.sqrt(hd)
    k = r.standard_normal((T, hd))
    v = r.standard_normal((T, hd))
    chunks = cp.zigzag_chunks(T, world, rank)
    q_chunks = [q[a:b] for a, b in chunks]
    k_chunks = [k[a:b] for a, b in chunks]
    v_chunks = [v[a:b] for a, b in chunks]

    def gather_kv(kc, vc):
        local = torch.from_numpy(np.stack(list(kc) + list(vc)))
        recv = [torch.empty_like(local) for _ in range(world)]
        work = dist.all_gather(recv, local, async_op=True)
        keys = np.full((T, hd), np.nan)
        values = np.full((T, hd), np.nan)

        def wait():
            work.wait()
            for rr in range(world):
                for i, (a, b) in enumerate(cp.zigzag_chunks(T, world, rr)):
                    keys[a:b] = recv[rr][i].numpy()
                    values[a:b] = recv[rr][2 + i].numpy()
        return wait, keys, values

    outs = cp.cp_prefill(q_chunks, k_chunks, v_chunks, T, world, rank, gather_kv, _np_attend, _np_merge)
    # reference: causal attention over the whole sequence for this rank's rows
    err = 0.0
    for (a, b), o in zip(chunks, outs):
        s = np.einsum("thd,kd->thk", q[a:b], k)
        s = np.where(np.arange(T)[None, None, :] <= np.arange(a, b)[:, None, None], s, -np.inf)
        s -= s.max(-1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(-1, keepdims=True)
        err = max(err, float(np.max(np.abs(p @ v - o))))
    first, second = cp.problems_for(T, world, rank)
    key_rows = sum(p.k1 - p.k0 for p in second)
    Path(result_dir, f"rank{rank}.txt").write_text(f"{err} {key_rows}")
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_cp_schedule_matches_causal_attention(tmp_path, world):
    import torch.multiprocessing as mp
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    T, hd = 64, 16
    mp.start_processes(_rank_main, args=(world, port, T, hd, str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    counts = []
    for rank in range(world):
        err, n = Path(tmp_path, f"rank{rank}.txt").read_text().split()
        assert float(err) < 1e-12, (rank, err)
        counts.append(int(n))
    # zigzag balance: every rank reads the same number of gathered key rows
    assert len(set(counts)) == 1


def test_zigzag_chunks_cover_the_sequence():
    sys.path.insert(0, str(ROOT / "gemma4-rs_b200"))
    from g4attn import cp
    for world in (1, 2, 4, 8):
        cov = sorted(c for r in range(world) for c in cp.zigzag_chunks(32768, world, r))
        assert cov[0][0] == 0 and cov[-1][1] == 32768
        assert all(cov[i][1] == cov[i + 1][0] for i in range(len(cov) - 1))
    with pytest.raises(ValueError):
        cp.zigzag_chunks(100, 8, 0)


class _NpKvShards:
    """The key/value-shard schedule's arithmetic in float64 numpy, its
    collectives over gloo (the reduce-scatter as an all-reduce and this
    rank's slice)."""

    def __init__(self, dist, torch, world, rank):
        self.dist, self.torch, self.world, self.rank = dist, torch, world, rank

    def attend(self, problems, q_all, k_chunks, v_chunks):
        from g4attn import cp
        probs = [cp.Problem(0, q0, q1, k0, k1, i) for i, (q0, q1, k0, k1) in enumerate(problems)]
        out = []
        for p in probs:
            out += _np_attend([p], [q_all[p.q0:p.q1]], lambda p: k_chunks[p.own], lambda p: v_chunks[p.own])
        return out

    def partial(self, seq_len, problems, results):
        (a0, _, _, _), (b0, _, _, _) = problems
        (oa, la), (ob, lb) = results
        hd = oa.shape[-1]
        o = np.zeros((seq_len, 8, hd))
        lse = np.full((seq_len, 8), -np.inf)
        o[a0:b0], lse[a0:b0] = oa[:b0 - a0], la[:b0 - a0]
        both = [(oa[b0 - a0:], la[b0 - a0:]), (ob, lb)]
        o[b0:] = _np_merge(both)
        m = np.maximum(both[0][1], both[1][1])
        lse[b0:] = m + np.log(np.exp(both[0][1] - m) + np.exp(both[1][1] - m))
        return o, lse

    def allreduce_max(self, lse):
        t = self.torch.from_numpy(lse.copy())
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return t.numpy()

    def weights(self, lse, m):
        return np.where(np.isfinite(lse), np.exp(np.where(np.isfinite(lse), lse - m, 0.0)), 0.0)

    def scale(self, o, w):
        return o * w[..., None]

    def to_rank_order(self, x, rows):
        return np.concatenate([x[a:b] for a, b in rows])

    def reduce_scatter_sum(self, x):
        t = self.torch.from_numpy(np.ascontiguousarray(x))
        self.dist.all_reduce(t, op=self.dist.ReduceOp.SUM)
        n = x.shape[0] // self.world
        return t.numpy()[self.rank * n:(self.rank + 1) * n]

    def finish(self, x, w):
        return x / w[..., None]


def _kv_shard_rank_main(rank, world, port, T, hd, result_dir):
    sys.path.insert(0, str(ROOT / "gemma4-rs_b200"))
    import torch
    import torch.distributed as dist
    from g4attn import cp
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    r = np.random.default_rng(9)
    q = r.standard_normal((T, 8, hd)) / np.sqrt(hd)
    k = r.standard_normal((T, hd))
    v = r.standard_normal((T, hd))
    chunks = cp.zigzag_chunks(T, world, rank)
    outs = cp.cp_prefill_kv_shards(q, [k[a:b] for a, b in chunks], [v[a:b] for a, b in chunks], T, world, rank,
                                   _NpKvShards(dist, torch, world, rank))
    err = 0.0
    for (a, b), o in zip(chunks, outs):
        s = np.einsum("thd,kd->thk", q[a:b], k)
        s = np.where(np.arange(T)[None, None, :] <= np.arange(a, b)[:, None, None], s, -np.inf)
        s -= s.max(-1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(-1, keepdims=True)
        err = max(err, float(np.max(np.abs(p @ v - o))))
    Path(result_dir, f"kv{rank}.txt").write_text(f"{err}")
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_kv_shard_schedule_matches_causal_attention(tmp_path, world):
    """Key/value shards and the cross-rank log-sum-exp merge (all-reduce of
    the maxima, reduce-scatter of the weighted partials): every rank's output
    chunks equal plain causal attention."""
    import torch.multiprocessing as mp
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    T, hd = 64, 16
    mp.start_processes(_kv_shard_rank_main, args=(world, port, T, hd, str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    for rank in range(world):
        assert float(Path(tmp_path, f"kv{rank}.txt").read_text()) < 1e-12, rank


def test_kv_shard_rows_cover_the_sequence():
    sys.path.insert(0, str(ROOT / "gemma4-rs_b200"))
    from g4attn import cp
    for world in (1, 2, 4, 8):
        rows = cp.rank_rows(1024, world)
        assert sorted(rows) == [(i * 1024 // (2 * world), (i + 1) * 1024 // (2 * world)) for i in range(2 * world)]
        for rank in range(world):
            probs = cp.kv_shard_problems(1024, world, rank)
            assert [p[2:] for p in probs] == cp.zigzag_chunks(1024, world, rank)
            assert all(p[0] == p[2] and p[1] == 1024 for p in probs)


# ---------------------------------------------------------------------------
# failures, made on the host: a rank that leaves, a rank that comes late, and
# ranks that disagree on the shard metadata
# ---------------------------------------------------------------------------

def _failure_rank_main(rank, world, port, mode, result_dir):
    sys.path.insert(0, str(ROOT / "gemma4-rs_b200"))
    import time
    from datetime import timedelta
    import torch
    import torch.distributed as dist
    from g4attn import cp
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    T, hd = 32, 8
    if mode == "disagree":
        T = 32 if rank == 0 else 48
    r = np.random.default_rng(3)
    q = r.standard_normal((T, 8, hd)) / np.sqrt(hd)
    k = r.standard_normal((T, hd))
    v = r.standard_normal((T, hd))
    t0 = time.monotonic()
    if mode == "dropped" and rank == world - 1:
        # this rank leaves between steps: it never enters the schedule
        Path(result_dir, f"f{rank}.txt").write_text("left")
        os._exit(0)
    if mode == "late" and rank == world - 1:
        time.sleep(1.0)  # well inside the group's 5 s timeout
    try:
        cp.check_agreement(dist, torch, seq_len=T, head_dim=hd)
        chunks = cp.zigzag_chunks(T, world, rank)
        outs = cp.cp_prefill_kv_shards(q, [k[a:b] for a, b in chunks], [v[a:b] for a, b in chunks], T, world,
                                       rank, _NpKvShards(dist, torch, world, rank))
        err = 0.0
        for (a, b), o in zip(chunks, outs):
            s = np.einsum("thd,kd->thk", q[a:b], k)
            s = np.where(np.arange(T)[None, None, :] <= np.arange(a, b)[:, None, None], s, -np.inf)
            s -= s.max(-1, keepdims=True)
            p = np.exp(s)
            p /= p.sum(-1, keepdims=True)
            err = max(err, float(np.max(np.abs(p @ v - o))))
        res = f"ok {err}"
    except ValueError as e:
        res = f"metadata {e}"
    except Exception as e:  # the collective failed: the peer is gone or timed out
        res = f"error {type(e).__name__}"
    Path(result_dir, f"f{rank}.txt").write_text(f"{res}|{time.monotonic() - t0:.2f}")
    os._exit(0)


def _run_failure(tmp_path, mode, world=2):
    import torch.multiprocessing as mp
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.start_processes(_failure_rank_main, args=(world, port, mode, str(tmp_path)), nprocs=world, join=False,
                             start_method="spawn")
    while not ctx.join(timeout=60):
        pass
    return [Path(tmp_path, f"f{r}.txt").read_text() for r in range(world)]


def test_cp_dropped_rank_raises_on_the_others(tmp_path):
    """A rank that leaves between steps: the remaining rank's first collective
    of the schedule fails with an error (no hang), within the group's
    timeout."""
    res = _run_failure(tmp_path, "dropped")
    assert res[1] == "left"
    what, secs = res[0].split("|")
    assert what.startswith("error"), res[0]
    assert float(secs) < 30.0


def test_cp_late_rank_still_agrees(tmp_path):
    """A rank that arrives a second late (inside the timeout): the schedule
    waits for it and every rank's result is still exact."""
    for r in _run_failure(tmp_path, "late"):
        what, _ = r.split("|")
        assert what.startswith("ok"), r
        assert float(what.split()[1]) < 1e-12


def test_cp_disagreeing_shard_metadata_is_rejected(tmp_path):
    """Ranks with different sequence lengths: every rank gets the metadata
    error before any data collective."""
    for r in _run_failure(tmp_path, "disagree"):
        what, _ = r.split("|")
        assert what.startswith("metadata ranks disagree on seq_len"), r
