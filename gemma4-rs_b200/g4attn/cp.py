"""Context-parallel prefill of a long global layer across ranks.

The reference has no multi-device code: it processes a prompt one token at a
time (crates/llm-gemma4/src/impl_/generate.rs:37-41), each position attending
to every earlier key on global layers (crates/llm-gemma4/src/eng/mod.rs:33-35).
Here the sequence is split over W ranks in 2W zigzag chunks: rank r holds the
queries and the keys/values of chunks r and 2W-1-r, which gives every rank the
same amount of causal work. With A = chunk r and B = chunk 2W-1-r, each rank

  1. starts an all-gather of the key/value chunks over NCCL on a side stream;
     the chunks land in one [T, hd] key and one value buffer in position order,
  2. meanwhile computes the two diagonal blocks A x A and B x B from its own
     chunks (g4a_prefill with position offsets, keeping each row's
     log-sum-exp),
  3. then A against keys [0, start of A) and B against keys [0, start of B)
     from the gathered buffers (one launch; every rank has (2W-1) chunks of
     keys in this phase),
  4. and merges the two partials of each query chunk by log-sum-exp
     (g4a_lse_merge).

Only the key/value chunks cross NVLink (2 x T x hd x 2 bytes in all); the
queries and outputs stay where they are.

The collective and merge schedule is written against three small callables so
that it can be checked on CPU ranks (gloo) with a numpy stand-in for the
attention arithmetic; the product path passes the CUDA library's functions.

The second schedule below (cp_prefill_kv_shards) keeps the keys and values
where they are and merges the ranks' partial outputs by log-sum-exp across
ranks (an all-reduce of the maxima, a reduce-scatter of the weighted sums).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Sequence


def zigzag_chunks(seq_len: int, world: int, rank: int) -> list[tuple[int, int]]:
    """The two [start, end) position ranges rank `rank` owns: chunks rank and
    2*world-1-rank of 2*world equal chunks."""
    n = 2 * world
    if seq_len % n:
        raise ValueError(f"sequence length {seq_len} is not a multiple of {n}")
    c = seq_len // n
    a, b = rank, n - 1 - rank
    return [(a * c, (a + 1) * c), (b * c, (b + 1) * c)]


def check_agreement(dist, torch, **meta: int) -> None:
    """Raises ValueError on every rank unless all ranks pass the same values
    (sequence length, head width, schedule ...): a rank with other shard
    metadata would make the collectives of the schedule exchange mismatched
    buffers. One small all-gather on the process group."""
    names = sorted(meta)
    mine = torch.tensor([int(meta[n]) for n in names], dtype=torch.int64)
    if dist.get_backend() == "nccl":
        mine = mine.cuda()
    every = [torch.empty_like(mine) for _ in range(dist.get_world_size())]
    dist.all_gather(every, mine)
    table = torch.stack(every).cpu()
    for i, n in enumerate(names):
        vals = table[:, i].tolist()
        if len(set(vals)) != 1:
            raise ValueError(f"ranks disagree on {n}: {vals}")


@dataclass
class Problem:
    """Queries [q0, q1) against keys [k0, k1) (absolute positions). own >= 0:
    the keys are this rank's chunk `own`; own < 0: rows [k0, k1) of the
    gathered buffers."""
    q_chunk: int   # index into this rank's query chunks (0 = A, 1 = B)
    q0: int
    q1: int
    k0: int
    k1: int
    own: int


def problems_for(seq_len: int, world: int, rank: int) -> tuple[list[Problem], list[Problem]]:
    """(before the gather, after the gather) problems of this rank."""
    (a0, a1), (b0, b1) = zigzag_chunks(seq_len, world, rank)
    first = [Problem(0, a0, a1, a0, a1, 0), Problem(1, b0, b1, b0, b1, 1)]
    second = ([Problem(0, a0, a1, 0, a0, -1)] if a0 > 0 else []) + [Problem(1, b0, b1, 0, b0, -1)]
    return first, second


def cp_prefill(q_chunks: Sequence, k_chunks: Sequence, v_chunks: Sequence, seq_len: int, world: int, rank: int,
               gather_kv: Callable, attend: Callable, merge: Callable):
    """Runs the schedule above.

    q_chunks/k_chunks/v_chunks: this rank's two chunks of queries [c, 8, hd]
    and keys/values [c, hd].
    gather_kv(k_chunks, v_chunks) -> (wait, keys, values): starts the
        all-gather; after wait(), keys[t] / values[t] hold position t's row.
    attend(problems, q_chunks, keys_of, values_of) -> list of (out, lse):
        partial attention for each Problem, keys_of(p) / values_of(p) giving
        its key/value rows.
    merge(parts) -> out: log-sum-exp merge of a query chunk's (out, lse) parts.
    Returns this rank's two output chunks.
    """
    first, second = problems_for(seq_len, world, rank)
    wait, keys, values = gather_kv(k_chunks, v_chunks)
    parts = [[], []]
    for p, r in zip(first, attend(first, q_chunks, lambda p: k_chunks[p.own], lambda p: v_chunks[p.own])):
        parts[p.q_chunk].append(r)
    wait()
    for p, r in zip(second, attend(second, q_chunks, lambda p: keys[p.k0:p.k1], lambda p: values[p.k0:p.k1])):
        parts[p.q_chunk].append(r)
    return [merge(parts[0]), merge(parts[1])]


# ---------------------------------------------------------------------------
# CUDA path: NCCL all-gather through torch.distributed, kernels from g4attn
# ---------------------------------------------------------------------------

def torch_gather_kv(dist, torch, side_stream):
    """All-gather of the key/value chunks on a side stream (NCCL), then a
    scatter of the chunks into position order on the caller's stream."""
    def gather(k_chunks, v_chunks):
        world = dist.get_world_size()
        c, hd = k_chunks[0].shape
        flat = torch.stack(list(k_chunks) + list(v_chunks))  # [4, c, hd]
        recv = torch.empty((world,) + tuple(flat.shape), dtype=flat.dtype, device=flat.device)
        keys = torch.empty(2 * world, c, hd, dtype=flat.dtype, device=flat.device)
        values = torch.empty_like(keys)
        main = torch.cuda.current_stream()
        side_stream.wait_stream(main)
        with torch.cuda.stream(side_stream):
            work = dist.all_gather_into_tensor(recv, flat, async_op=True)

        def wait():
            work.wait()
            main.wait_stream(side_stream)
            recv.record_stream(main)
            # rank r's chunk 0 is chunk r, its chunk 1 is chunk 2W-1-r
            keys[:world].copy_(recv[:, 0])
            keys[world:].copy_(recv[:, 1].flip(0))
            values[:world].copy_(recv[:, 2])
            values[world:].copy_(recv[:, 3].flip(0))
        return wait, keys.view(-1, hd), values.view(-1, hd)
    return gather


def g4a_attend(ctx, torch, head_dim: int):
    """Partial attention of several Problems in one g4a_prefill launch."""
    def attend(problems, q_chunks, keys_of, values_of):
        outs = []
        specs = []
        for p in problems:
            n_q = p.q1 - p.q0
            out = torch.empty(n_q, 8, head_dim, device="cuda")
            lse = torch.empty(n_q, 8, device="cuda")
            specs.append(dict(head_dim=head_dim, window=0, n_q=n_q, q_pos0=p.q0, n_kv=p.k1 - p.k0, kv_pos0=p.k0,
                              q=q_chunks[p.q_chunk], k=keys_of(p), v=values_of(p), out=out, lse=lse))
            outs.append((out, lse))
        ctx.prefill(specs)
        return outs
    return attend


def g4a_merge(ctx, torch, head_dim: int):
    """Log-sum-exp merge on the device; g4a_lse_merge takes up to 16 parts at
    a time, so longer lists are folded in rounds."""
    def merge(parts):
        parts = list(parts)
        if len(parts) == 1:
            return parts[0][0]
        rows = parts[0][0].shape[0]
        while len(parts) > 1:
            batch, parts = parts[:16], parts[16:]
            o = torch.empty_like(batch[0][0])
            l = torch.empty(rows, 8, device=o.device)
            ctx.lse_merge([b[0] for b in batch], [b[1] for b in batch], rows, 8, head_dim, o, l)
            parts = [(o, l)] + parts
        return parts[0][0]
    return merge


# ---------------------------------------------------------------------------
# Key/value shards with a cross-rank log-sum-exp merge
# ---------------------------------------------------------------------------
#
# The other partition of the same problem: each rank keeps only its own key/
# value chunks (the zigzag pair above, so that causal work stays balanced)
# and attends every query that sees them. Per rank and query row that gives a
# normalized partial output O_r and its log-sum-exp l_r (rows that see none of
# the rank's keys: O_r = 0, l_r = -inf). Then
#
#   M   = max over ranks of l_r          (all-reduce, MAX, [T, heads])
#   w_r = exp(l_r - M)                   (0 where l_r = -inf)
#   O   = sum_r w_r O_r / sum_r w_r       (reduce-scatter, SUM, of w_r O_r and
#                                         w_r: each rank receives the rows of
#                                         its own two query chunks)
#
# No key/value row leaves its rank; the queries are all-gathered first and
# the partial outputs (f32, all rows) cross the links once, so this moves
# about 2 x T x heads x hd x 4 bytes per rank against the all-gather
# schedule's 2 x T x hd x 2 in all.


def kv_shard_problems(seq_len: int, world: int, rank: int) -> list[tuple[int, int, int, int]]:
    """(q0, q1, k0, k1) for each of this rank's two key chunks: every query at
    or after the chunk's first position sees it (causal)."""
    return [(k0, seq_len, k0, k1) for k0, k1 in zigzag_chunks(seq_len, world, rank)]


def rank_rows(seq_len: int, world: int) -> list[tuple[int, int]]:
    """Row ranges in the order a reduce-scatter hands them out: rank 0's two
    query chunks, then rank 1's, ..."""
    return [c for r in range(world) for c in zigzag_chunks(seq_len, world, r)]


def cp_prefill_kv_shards(q_all, k_chunks: Sequence, v_chunks: Sequence, seq_len: int, world: int, rank: int, be):
    """Runs the key/value-shard schedule on one rank.

    q_all: [T, heads, hd] queries (every rank's, as gathered); k_chunks /
    v_chunks: this rank's two key/value chunks [c, hd].
    be: the arithmetic and collectives, with
      attend(problems, q_all, k_chunks, v_chunks) -> [(out [n, heads, hd], lse [n, heads])]
          (problem i uses key chunk i);
      partial(seq_len, problems, results) -> (O [T, heads, hd], lse [T, heads]):
          this rank's two results on all rows, merged where both apply;
      allreduce_max(lse) -> M;  weights(lse, M) -> exp(lse - M), 0 at -inf;
      scale(O, w) -> w O;  to_rank_order(x, rows) -> x's row ranges `rows`
          concatenated;  reduce_scatter_sum(x) -> this rank's 2c rows of the
          sum over ranks;  finish(X, w) -> X / w.
    Returns this rank's two output chunks [c, heads, hd] (chunks r and
    2W-1-r)."""
    problems = kv_shard_problems(seq_len, world, rank)
    results = be.attend(problems, q_all, k_chunks, v_chunks)
    o_r, lse_r = be.partial(seq_len, problems, results)
    m = be.allreduce_max(lse_r)
    w = be.weights(lse_r, m)
    rows = rank_rows(seq_len, world)
    x = be.reduce_scatter_sum(be.to_rank_order(be.scale(o_r, w), rows))
    ws = be.reduce_scatter_sum(be.to_rank_order(w, rows))
    out = be.finish(x, ws)
    c = seq_len // (2 * world)
    return [out[:c], out[c:]]


class TorchKvShardBackend:
    """The key/value-shard schedule on the GPU: g4a_prefill for the partial
    attention (with position offsets and the log-sum-exp), g4a_lse_merge for
    the rank's own two partials, NCCL through torch.distributed for the
    all-reduce and the reduce-scatter, elementwise weights in torch."""

    def __init__(self, ctx, torch, dist, head_dim: int, heads: int = 8):
        self.ctx, self.torch, self.dist, self.hd, self.heads = ctx, torch, dist, head_dim, heads

    def attend(self, problems, q_all, k_chunks, v_chunks):
        torch, specs, outs = self.torch, [], []
        for i, (q0, q1, k0, k1) in enumerate(problems):
            out = torch.empty(q1 - q0, self.heads, self.hd, device=q_all.device)
            lse = torch.empty(q1 - q0, self.heads, device=q_all.device)
            specs.append(dict(head_dim=self.hd, window=0, n_q=q1 - q0, q_pos0=q0, n_kv=k1 - k0, kv_pos0=k0,
                              q=q_all[q0:q1], k=k_chunks[i], v=v_chunks[i], out=out, lse=lse))
            outs.append((out, lse))
        self.ctx.prefill(specs)
        return outs

    def partial(self, seq_len, problems, results):
        torch = self.torch
        (a0, _, _, _), (b0, _, _, _) = problems
        (oa, la), (ob, lb) = results
        o = torch.zeros(seq_len, self.heads, self.hd, device=oa.device)
        lse = torch.full((seq_len, self.heads), float("-inf"), device=oa.device)
        o[a0:b0] = oa[:b0 - a0]
        lse[a0:b0] = la[:b0 - a0]
        n = seq_len - b0  # rows that see both chunks
        o_both, l_both = o[b0:], lse[b0:]
        self.ctx.lse_merge([oa[b0 - a0:].contiguous(), ob], [la[b0 - a0:].contiguous(), lb], n, self.heads, self.hd,
                           o_both, l_both)
        return o, lse

    def allreduce_max(self, lse):
        m = lse.clone()
        self.dist.all_reduce(m, op=self.dist.ReduceOp.MAX)
        return m

    def weights(self, lse, m):
        torch = self.torch
        return torch.where(torch.isfinite(lse), torch.exp(lse - m), torch.zeros_like(lse))

    def scale(self, o, w):
        return o * w[..., None]

    def to_rank_order(self, x, rows):
        return self.torch.cat([x[a:b] for a, b in rows]).contiguous()

    def reduce_scatter_sum(self, x):
        world = self.dist.get_world_size()
        out = self.torch.empty((x.shape[0] // world,) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
        self.dist.reduce_scatter_tensor(out, x, op=self.dist.ReduceOp.SUM)
        return out

    def finish(self, x, w):
        return x / w[..., None]
