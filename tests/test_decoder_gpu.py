"""The E2B decoder on the GPU (g4a_model_*) against the oracle's restatement
of crates/llm-gemma4/src/impl_/model.rs:252-449 and generate.rs:15-64, on
seeded synthetic weights in the GGUF layout (config 4's model, the vocabulary
reduced where the oracle would spend minutes on the head).

The reference's bar is the same top-1 token at every step. On this random
model that needs every bit: one last-place difference in an activation can
cross a Q8_0 rounding boundary of the next projection's input, and the
model's sharp attention (unit-RMS q and k, no 1/sqrt(d) scale) carries it to
different greedy tokens within a few layers. So the device computes what the
reference computes, in its order (integer block dots, attention in
attend_head's order, glibc's expf and tanhf restated), and the bar here is
bit-identical logits and tokens. Both engines consume the same tokens (the
device's picks) so every step is compared on equal inputs.
"""
import os

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
    c = g4attn.Context(0, max_positions=4096)
    yield c
    c.close()


def host_decoder(oracle, w):
    import g4attn.model as gm
    host = {name: w.host(name) for name in w.tensors}
    return lambda: oracle.Decoder(w.hp, host, w.d_model, w.vocab, w.ple_dim, w.d_ff, w.softcap, gm.rope_freqs(w.hp),
                                  w.scales)


@pytest.fixture(scope="module")
def small_vocab(ctx, oracle):
    import g4attn.model as gm
    oracle.pool_init(min(32, os.cpu_count() or 1))
    w = gm.synthetic_weights(ctx, vocab=4096, seed=11)
    return w, host_decoder(oracle, w)


def compare_step(got_logits, want_logits, got_tok, stats, oracle):
    diff = float(np.max(np.abs(got_logits.astype(np.float64) - want_logits)))
    stats["max_diff"] = max(stats["max_diff"], diff)
    stats["bit_identical"] += int(np.array_equal(got_logits.view(np.uint32), want_logits.view(np.uint32)))
    stats["top1_agree"] += int(got_tok == oracle.argmax_total(want_logits))
    stats["steps"] += 1


def check(stats):
    assert stats["bit_identical"] == stats["steps"] and stats["top1_agree"] == stats["steps"], stats


def synth_normals(seed: int, tensor: int, n: int) -> np.ndarray:
    """Host restatement of the device generator's N(0, 1) stream (splitmix64
    finaliser of a counter, Box-Muller on two 24-bit uniforms)."""
    M = (1 << 64) - 1

    def mix(z):
        z = (z + 0x9E3779B97F4A7C15) & M
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M
        return z ^ (z >> 31)
    out = np.empty(n)
    for i in range(n):
        h = mix(seed ^ mix((tensor * 0x100000001B3 + i) & M))
        u1 = ((h >> 40) + 1) / 16777216.0
        u2 = (h & 0xFFFFFF) / 16777216.0
        out[i] = np.sqrt(-2 * np.log(u1)) * np.cos(2 * np.pi * u2)
    return out


def test_synthetic_weights_layout(ctx, small_vocab):
    """Q8_0 blocks as a GGUF file holds them: f16 scale = max|w|/127, so each
    block's largest |quant| is 127; values ~ N(0, 0.02); seeded; the bytes
    are the host restatement's (device logf/cospif may move a rare value
    across a rounding boundary)."""
    import g4attn.model as gm
    w, _ = small_vocab
    b = w.host("blk.0.attn_q.weight").reshape(-1, 34)
    ref = (0.02 * synth_normals(11, gm.fnv1a64("blk.0.attn_q.weight"), 64 * 32)).astype(np.float32).reshape(64, 32)
    ref_scale = (np.abs(ref).max(1) / np.float32(127)).astype(np.float32)
    ref_q = np.clip(np.round(ref / ref_scale[:, None]), -128, 127).astype(np.int8)
    got_scale = b[:64, :2].copy().view(np.float16).ravel()
    assert np.mean(got_scale == ref_scale.astype(np.float16)) >= 0.95, (b[:4, :2], ref_scale[:4].astype(np.float16))
    assert np.mean(b[:64, 2:].view(np.int8) == ref_q) >= 0.99
    scales = b[:, :2].copy().view(np.float16).astype(np.float32).ravel()
    quants = b[:, 2:].view(np.int8)
    assert np.all(np.abs(quants).max(axis=1) == 127)
    vals = (quants.astype(np.float32) * scales[:, None]).ravel()
    assert abs(vals.std() - 0.02) < 0.001 and abs(vals.mean()) < 0.001
    again = gm.synthetic_weights(ctx, vocab=64, seed=11, ple_dim=0)
    assert np.array_equal(again.host("blk.0.attn_q.weight"), w.host("blk.0.attn_q.weight"))
    n = w.host("blk.3.ffn_norm.weight")
    assert np.array_equal(n, n.astype(np.float32).view(np.uint32).__and__(0xFFFF0000).view(np.float32))  # bf16


def test_steps_match_oracle(ctx, small_vocab, oracle):
    """Three sequences in one batch at different positions (one joins late),
    through the eager first step, the graph capture and graph replays; past
    the 512-row window is config 2's job, here every layer's full causal
    range and the window policy's lower bound of 0 are exercised."""
    import g4attn.model as gm
    w, make = small_vocab
    m = gm.Model(ctx, w, max_seqs=4, max_tokens=128)
    decs = [make() for _ in range(3)]
    r = rng(12)
    prompts = [list(r.integers(0, w.vocab, 19)) for _ in range(3)]
    pos = [0, 0, 0]
    cur = [int(prompts[i][0]) for i in range(3)]
    stats = {"max_diff": 0.0, "bit_identical": 0, "top1_agree": 0, "steps": 0}
    for step in range(40):
        ids = [0, 2] if step < 6 else [0, 2, 3]  # sequence 3 starts at step 6
        rows = [0, 1] if step < 6 else [0, 1, 2]
        toks = [cur[i] for i in rows]
        nxt = m.step(ids, toks)
        logits = m.logits().cpu().numpy()
        for j, i in enumerate(rows):
            want = decs[i].forward(toks[j], pos[i])
            compare_step(logits[j], want, nxt[j], stats, oracle)
            pos[i] += 1
            cur[i] = int(prompts[i][pos[i]]) if pos[i] < 19 else nxt[j]
    assert [m.len(s) for s in (0, 2, 3)] == [pos[0], pos[1], pos[2]]
    print(f"decoder steps vs oracle: {stats}")
    check(stats)
    m.close()


def test_batched_steps_match_oracle(ctx, small_vocab, oracle):
    """Twelve sequences per step: the batched path (tensor-core Q8_0 GEMMs,
    separate residual kernels), bit-identical to the oracle too."""
    import g4attn.model as gm
    w, make = small_vocab
    n = 12
    m = gm.Model(ctx, w, max_seqs=n, max_tokens=32)
    decs = [make() for _ in range(n)]
    toks = rng(15).integers(0, w.vocab, (n, 6))
    stats = {"max_diff": 0.0, "bit_identical": 0, "top1_agree": 0, "steps": 0}
    cur = [int(t) for t in toks[:, 0]]
    for p in range(8):
        nxt = m.step(list(range(n)), cur)
        logits = m.logits().cpu().numpy()
        for i in range(n):
            compare_step(logits[i], decs[i].forward(cur[i], p), nxt[i], stats, oracle)
        cur = [int(toks[i, p + 1]) if p + 1 < 6 else nxt[i] for i in range(n)]
    print(f"batched steps vs oracle: {stats}")
    check(stats)
    m.close()


def test_long_cache_split_attention(ctx, small_vocab, oracle):
    """Caches longer than the exact attention's 4096 rows take the split-KV
    decode kernel (within the decode tolerance of 1e-4, not bit-exact). While
    the attention spans one to three rows its output is exact or nearly so
    and the logits match the oracle's; later, on this random model, a
    last-place difference can flip a Q8_0 rounding and the logits drift
    (reported), staying finite and inside the soft-cap."""
    import g4attn
    import g4attn.model as gm
    w, make = small_vocab
    ctx8 = g4attn.Context(0, max_positions=4200)
    m = gm.Model(ctx8, w, max_seqs=2, max_tokens=4160)
    dec = make()
    toks = [int(t) for t in rng(16).integers(0, w.vocab, 12)]
    diffs = []
    for p, tok in enumerate(toks):
        m.step([1], [tok])
        got = m.logits().cpu().numpy()[0].astype(np.float64)
        want = dec.forward(tok, p).astype(np.float64)
        diffs.append(float(np.max(np.abs(got - want))))
        assert np.all(np.isfinite(got)) and np.all(np.abs(got) <= 30.0)
    print(f"split-KV path, max |logit diff| per step: {[f'{d:.1e}' for d in diffs]}")
    assert max(diffs[:3]) <= 1e-3
    m.close()
    ctx8.close()


def test_generate_matches_oracle(ctx, small_vocab):
    """g4a_model_generate (generate.rs:15-64, greedy) against the oracle's
    generate, token for token."""
    import g4attn.model as gm
    w, make = small_vocab
    m = gm.Model(ctx, w, max_seqs=2, max_tokens=64)
    prompts = rng(13).integers(0, w.vocab, (2, 19)).astype(np.int32)
    out = m.generate(prompts, 12)
    for i in range(2):
        assert out[i].tolist() == make().generate(prompts[i].tolist(), 12)
    m.close()


def test_generate_stops_at_eos(ctx, small_vocab):
    """With eos_token_ids set, a sequence keeps its eos token and stops
    (generate.rs:58-60) while the others go on; each row is the oracle's
    generate with the same eos, then -1."""
    import g4attn.model as gm
    w, make = small_vocab
    m = gm.Model(ctx, w, max_seqs=3, max_tokens=64)
    prompts = rng(23).integers(0, w.vocab, (3, 11)).astype(np.int32)
    free = m.generate(prompts, 14)
    eos = [int(free[0, 5]), int(free[1, 9])]
    m.set_eos(eos)
    out = m.generate(prompts, 14)
    stopped = 0
    for i in range(3):
        want = make().generate(prompts[i].tolist(), 14, eos=tuple(eos))
        assert out[i, :len(want)].tolist() == want, i
        assert np.all(out[i, len(want):] == -1), i
        stopped += len(want) < 14
    assert stopped >= 2
    m.set_eos([])
    assert np.array_equal(m.generate(prompts, 14), free)
    m.close()


def test_prefill_chunks_match_steps_and_oracle(ctx, small_vocab, oracle, monkeypatch):
    """g4a_model_prefill in chunks of many positions (rows bounded to 14 here,
    so two prompts go through as chunks of 7, 7, ..., 5 positions, and one
    prompt continues a sequence that already holds 5 tokens): the caches
    are bit-identical to token-by-token steps of the same tokens, and the
    logits after each prompt and of the steps that follow are the oracle's
    bit for bit."""
    import g4attn.model as gm
    w, make = small_vocab
    monkeypatch.setenv("G4A_CHUNK_ROWS", "14")
    m = gm.Model(ctx, w, max_seqs=4, max_tokens=96)
    r = rng(17)
    p0, p1 = r.integers(0, w.vocab, 40).astype(np.int32), r.integers(0, w.vocab, 40).astype(np.int32)
    head = [int(t) for t in r.integers(0, w.vocab, 5)]
    for t in head:  # sequence 1 holds 5 tokens before its prompt
        m.step([1], [t])
    nxt = m.prefill([0, 1], np.stack([p0, p1]))
    assert [m.len(0), m.len(1)] == [40, 45]
    got = m.logits().cpu().numpy()
    decs = [make(), make()]
    seqs = [p0.tolist(), head + p1.tolist()]
    stats = {"max_diff": 0.0, "bit_identical": 0, "top1_agree": 0, "steps": 0}
    for i in range(2):
        for p, t in enumerate(seqs[i][:-1]):
            decs[i].forward(t, p)
        compare_step(got[i], decs[i].forward(seqs[i][-1], len(seqs[i]) - 1), nxt[i], stats, oracle)
    # the same tokens step by step in sequences 2 and 3: the same K/V rows
    for t in p0:
        m.step([2], [int(t)])
    for t in seqs[1]:
        m.step([3], [int(t)])
    for layer in (0, 4, 13, 14):
        for a, b, n in ((0, 2, 40), (1, 3, 45)):
            ka, va = m.kv_view(a, layer, n)
            kb, vb = m.kv_view(b, layer, n)
            assert ka.cpu().numpy().tobytes() == kb.cpu().numpy().tobytes(), (layer, a)
            assert va.cpu().numpy().tobytes() == vb.cpu().numpy().tobytes(), (layer, a)
    # decoding continues from the chunked caches
    cur = list(nxt)
    for _ in range(6):
        nxt = m.step([0, 1], cur)
        logits = m.logits().cpu().numpy()
        for i in range(2):
            compare_step(logits[i], decs[i].forward(cur[i], m.len(i) - 1), nxt[i], stats, oracle)
        cur = list(nxt)
    print(f"chunked prefill vs oracle: {stats}")
    check(stats)
    m.close()


def test_prefill_one_position_chunks(ctx, small_vocab, monkeypatch):
    """Rows for only one position per sequence: each chunk is a decode step
    (its captured graph); the tokens are those of the many-position chunks."""
    import g4attn.model as gm
    w, _ = small_vocab
    prompts = rng(18).integers(0, w.vocab, (3, 9)).astype(np.int32)
    monkeypatch.setenv("G4A_CHUNK_ROWS", "4")
    m1 = gm.Model(ctx, w, max_seqs=3, max_tokens=16)
    a = m1.prefill([0, 1, 2], prompts)
    la = m1.logits().cpu().numpy()
    m1.close()
    monkeypatch.delenv("G4A_CHUNK_ROWS")
    m2 = gm.Model(ctx, w, max_seqs=3, max_tokens=16)
    b = m2.prefill([2, 0, 1], prompts[[2, 0, 1]])
    lb = m2.logits().cpu().numpy()
    m2.close()
    assert a == [b[1], b[2], b[0]]
    assert la.tobytes() == lb[[1, 2, 0]].tobytes()


def test_prefill_past_the_window(ctx, small_vocab, oracle):
    """A 600-token prompt in one chunk: the local layers' rows attend their
    512-row window (eng/mod.rs:10-36), the global ones all rows; the logits
    after the prompt and of the next steps are the oracle's bit for bit."""
    import g4attn.model as gm
    w, make = small_vocab
    m = gm.Model(ctx, w, max_seqs=1, max_tokens=640)
    prompt = rng(19).integers(0, w.vocab, 600).astype(np.int32)
    nxt = m.prefill([0], prompt[None, :])[0]
    dec = make()
    for p, t in enumerate(prompt[:-1].tolist()):
        dec.forward(t, p)
    stats = {"max_diff": 0.0, "bit_identical": 0, "top1_agree": 0, "steps": 0}
    compare_step(m.logits().cpu().numpy()[0], dec.forward(int(prompt[-1]), 599), nxt, stats, oracle)
    for p in range(600, 603):
        tok = nxt
        nxt = m.step([0], [tok])[0]
        compare_step(m.logits().cpu().numpy()[0], dec.forward(tok, p), nxt, stats, oracle)
    print(f"600-token prefill vs oracle: {stats}")
    check(stats)
    m.close()


def test_full_e2b_top1(ctx, oracle):
    """Config 4's model at full size (vocab 262,144, 3.9 GB of Q8_0 weights):
    a 19-token prompt and greedy steps, logits against the oracle."""
    import g4attn.model as gm
    w = gm.synthetic_weights(ctx, seed=4)
    assert w.vocab == 262_144 and w.d_model == 1536 and w.d_ff == 3072
    make = host_decoder(oracle, w)
    m = gm.Model(ctx, w, max_seqs=1, max_tokens=64)
    dec = make()
    prompt = [int(t) for t in rng(14).integers(0, w.vocab, 19)]
    stats = {"max_diff": 0.0, "bit_identical": 0, "top1_agree": 0, "steps": 0}
    tok = prompt[0]
    for p in range(24):
        nxt = m.step([0], [tok])[0]
        compare_step(m.logits().cpu().numpy()[0], dec.forward(tok, p), nxt, stats, oracle)
        tok = prompt[p + 1] if p + 1 < 19 else nxt
    print(f"full E2B vs oracle: {stats}")
    check(stats)
    m.close()


def test_errors(ctx, small_vocab, torch_cuda):
    import g4attn
    import g4attn.model as gm
    w, _ = small_vocab
    m = gm.Model(ctx, w, max_seqs=2, max_tokens=3)
    with pytest.raises(g4attn.EngError) as e:
        m.step([0], [w.vocab])
    assert e.value.code == g4attn.COMPUTE and "exceeds vocabulary" in e.value.message
    with pytest.raises(g4attn.EngError) as e:
        m.step([1, 1], [0, 0])
    assert e.value.code == g4attn.COMPUTE
    for _ in range(3):
        m.step([0], [5])
    with pytest.raises(g4attn.EngError) as e:
        m.step([0], [5])
    assert e.value.code == g4attn.CONTEXT_TOO_LONG and "got 4, max 3" in e.value.message
    assert m.len(0) == 3
    m.clear(0)
    assert m.len(0) == 0
    m.step([0], [5])
    with pytest.raises(g4attn.EngError) as e:
        m.generate(np.zeros((1, 5), np.int32), 2, max_context=4)
    assert e.value.code == g4attn.CONTEXT_TOO_LONG
    m.clear(0)
    with pytest.raises(g4attn.EngError) as e:  # a prompt past the capacity: nothing runs
        m.prefill([0], np.zeros((1, 4), np.int32))
    assert e.value.code == g4attn.CONTEXT_TOO_LONG and "got 4, max 3" in e.value.message
    with pytest.raises(g4attn.EngError) as e:
        m.prefill([0], np.full((1, 2), w.vocab, np.int32))
    assert e.value.code == g4attn.COMPUTE and "exceeds vocabulary" in e.value.message
    with pytest.raises(g4attn.EngError) as e:
        m.prefill([0, 0], np.zeros((2, 2), np.int32))
    assert e.value.code == g4attn.COMPUTE
    assert m.len(0) == 0
    m.prefill([0], np.zeros((1, 3), np.int32))
    assert m.len(0) == 3
    m.close()
    missing = gm.Weights(w.hp, w.vocab, w.d_model, w.d_ff, w.ple_dim, w.softcap)
    missing.tensors = dict(w.tensors)
    del missing.tensors["blk.7.ffn_up.weight"]
    with pytest.raises(g4attn.EngError) as e:
        gm.Model(ctx, missing, 1, 8)
    assert e.value.code == g4attn.MISSING_WEIGHT and "blk.7.ffn_up.weight" in e.value.message


def test_box_libm_matches_restatement(tmp_path):
    """The oracle on this machine calls its C library's expf/tanhf; the device
    restates glibc's. Check that this machine's library is that one."""
    from test_libm_restatement import run_check
    bad, checked = run_check(tmp_path)
    assert bad == 0, (bad, checked)
