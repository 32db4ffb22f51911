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
