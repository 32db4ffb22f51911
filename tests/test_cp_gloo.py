"""Context-parallel prefill schedule on CPU ranks (gloo, world size 2 and 4):
zigzag chunking, the key/value all-gather, which (query, key) chunk pairs each
rank computes, and the log-sum-exp merge, with a float64 numpy stand-in for
the attention arithmetic. The result must equal plain causal attention."""
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
