"""The oracle's E2B decoder (orc_dec_forward, a C restatement of
crates/llm-gemma4/src/impl_/model.rs:252-449) on a small synthetic model.

Pins: (1) its composition equals a step-by-step Python composition of the
oracle's own pinned primitives (rms_norm, quantize/matvec Q8_0, the attention
block, gelu, soft-cap) bit for bit; (2) the reference's synthetic_generate.rs
properties: incremental decoding equals recomputing the whole prefix, and a
token's logits do not depend on later tokens; (3) generate follows
generate.rs:15-64 (prompt tokens fed one at a time, greedy samples, the last
one not fed back).
"""
import numpy as np
import pytest

from helpers import rng

D, DFF, PLE, VOCAB = 128, 256, 32, 97


def tiny_hp(oracle):
    hp = oracle.HParams()
    oracle.lib().orc_hparams_e2b(hp)
    hp.n_layers, hp.head_dim_local, hp.head_dim_global = 7, 64, 128
    hp.sliding_window, hp.shared_kv_layers = 16, 2  # layers 5 (local) and 6 (global) share KV
    return hp


def tiny_weights(oracle, hp, seed=0):
    r = rng(seed)
    w = {}

    def q8(name, rows, cols):
        w[name] = oracle.q8_0_bytes_of(r.standard_normal(rows * cols).astype(np.float32) * 0.05)

    def norm(name, n):
        w[name] = np.array([oracle.lib().orc_round_bf16(float(v)) for v in 1.0 + 0.1 * r.standard_normal(n)],
                           np.float32)

    q8("token_embd.weight", VOCAB, D)
    norm("output_norm.weight", D)
    q8("per_layer_token_embd.weight", VOCAB, hp.n_layers * PLE)
    q8("per_layer_model_proj.weight", hp.n_layers * PLE, D)
    norm("per_layer_proj_norm.weight", PLE)
    scales = {}
    for l in range(hp.n_layers):
        hd = oracle.head_dim(hp, l)
        b = f"blk.{l}."
        for n in ("attn_norm", "post_attention_norm", "ffn_norm", "post_ffw_norm", "post_norm"):
            norm(b + n + ".weight", D)
        norm(b + "attn_q_norm.weight", hd)
        norm(b + "attn_k_norm.weight", hd)
        q8(b + "attn_q.weight", 8 * hd, D)
        q8(b + "attn_k.weight", hd, D)
        q8(b + "attn_v.weight", hd, D)
        q8(b + "attn_output.weight", D, 8 * hd)
        q8(b + "ffn_gate.weight", DFF, D)
        q8(b + "ffn_up.weight", DFF, D)
        q8(b + "ffn_down.weight", D, DFF)
        q8(b + "inp_gate.weight", PLE, D)
        q8(b + "proj.weight", D, PLE)
        scales[l] = float(np.float32(1.0 + 0.1 * r.standard_normal()))
    return w, scales


@pytest.fixture(scope="module")
def tiny(oracle):
    hp = tiny_hp(oracle)
    w, scales = tiny_weights(oracle, hp)
    freqs = oracle.proportional_rope_freq_factors(hp.head_dim_global, hp.global_p)
    return hp, w, scales, freqs


def decoder(oracle, tiny):
    hp, w, scales, freqs = tiny
    return oracle.Decoder(hp, w, D, VOCAB, PLE, DFF, 30.0, freqs, scales)


def project(oracle, w, rows, x):
    s, q = oracle.quantize_q8_0(x)
    return oracle.matvec_q8_0(w, rows, len(x), s, q)


def python_forward(oracle, tiny, kv, token, position):
    """model.rs:376-449 composed in Python from the oracle's primitives."""
    hp, w, scales, freqs = tiny
    eps, L = hp.rms_norm_eps, hp.n_layers
    row = lambda name, i, cols: oracle.dequant_q8_0(w[name].reshape(-1, cols // 32 * 34)[i])
    x = row("token_embd.weight", token, D) * np.float32(np.sqrt(np.float32(D)))
    projected = project(oracle, w["per_layer_model_proj.weight"], L * PLE, x)
    table = row("per_layer_token_embd.weight", token, L * PLE)
    ps, ts, is_ = np.float32(1) / np.sqrt(np.float32(D)), np.sqrt(np.float32(PLE)), np.float32(1) / np.sqrt(np.float32(2))
    pli = []
    for l in range(L):
        normed = oracle.rms_norm(projected[l * PLE:(l + 1) * PLE] * ps, w["per_layer_proj_norm.weight"], eps)
        pli.append((normed + table[l * PLE:(l + 1) * PLE] * ts) * is_)
    for l in range(L):
        b = f"blk.{l}."
        hd = oracle.head_dim(hp, l)
        src, _ = oracle.kv_source_layer(hp, l)
        n = oracle.rms_norm(x, w[b + "attn_norm.weight"], eps)
        q = project(oracle, w[b + "attn_q.weight"], 8 * hd, n)
        k = v = None
        if src == l:
            k = project(oracle, w[b + "attn_k.weight"], hd, n)
            v = project(oracle, w[b + "attn_v.weight"], hd, n)
        att = kv.attention_block(hp, l, position, q, k, v, w[b + "attn_q_norm.weight"], w[b + "attn_k_norm.weight"],
                                 freqs)
        a = oracle.rms_norm(project(oracle, w[b + "attn_output.weight"], D, att), w[b + "post_attention_norm.weight"],
                            eps)
        x = x + a
        n = oracle.rms_norm(x, w[b + "ffn_norm.weight"], eps)
        s, qq = oracle.quantize_q8_0(n)
        gated = oracle.geglu_q8_0(w[b + "ffn_gate.weight"], w[b + "ffn_up.weight"], DFF, D, s, qq)
        x = x + oracle.rms_norm(project(oracle, w[b + "ffn_down.weight"], D, gated), w[b + "post_ffw_norm.weight"], eps)
        gate = project(oracle, w[b + "inp_gate.weight"], PLE, x)
        g = oracle.gelu_tanh(gate) * pli[l]
        x = x + oracle.rms_norm(project(oracle, w[b + "proj.weight"], D, g), w[b + "post_norm.weight"], eps)
        x = x * np.float32(scales[l])
    n = oracle.rms_norm(x, w["output_norm.weight"], eps)
    s, qq = oracle.quantize_q8_0(n)
    return oracle.matvec_q8_0_softcap(w["token_embd.weight"], VOCAB, D, s, qq, 30.0)


def test_forward_equals_python_composition(oracle, tiny):
    dec = decoder(oracle, tiny)
    kv = oracle.KvCache()
    tokens = rng(5).integers(0, VOCAB, 24)
    for pos, t in enumerate(tokens):  # past the 16-row window
        got = dec.forward(int(t), pos)
        want = python_forward(oracle, tiny, kv, int(t), pos)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), pos
        assert np.all(np.abs(got) <= 30.0) and np.all(np.isfinite(got))


def test_incremental_equals_recompute_and_causal(oracle, tiny):
    """synthetic_generate.rs:36-72: cached decoding equals recomputing the
    prefix; logits of a position do not change with later tokens."""
    tokens = [int(t) for t in rng(6).integers(0, VOCAB, 20)]
    dec = decoder(oracle, tiny)
    incremental = [dec.forward(t, p) for p, t in enumerate(tokens)]
    for cut in (1, 7, 17, 20):
        fresh = decoder(oracle, tiny)
        for p, t in enumerate(tokens[:cut]):
            last = fresh.forward(t, p)
        assert np.array_equal(last, incremental[cut - 1])
    other = decoder(oracle, tiny)
    changed = tokens[:10] + [(t + 1) % VOCAB for t in tokens[10:]]
    for p, t in enumerate(changed):
        got = other.forward(t, p)
        if p < 10:
            assert np.array_equal(got, incremental[p])


def test_generate_greedy_loop(oracle, tiny):
    prompt = [int(t) for t in rng(7).integers(0, VOCAB, 5)]
    dec = decoder(oracle, tiny)
    out = dec.generate(prompt, 6)
    # by hand: the prompt, then each sample fed back except the last
    ref = decoder(oracle, tiny)
    logits = None
    for p, t in enumerate(prompt):
        logits = ref.forward(t, p)
    want = []
    for i in range(6):
        want.append(oracle.argmax_total(logits))
        if i < 5:
            logits = ref.forward(want[-1], len(prompt) + i)
    assert out == want and len(out) == 6


def test_generate_eos_stops(oracle, tiny):
    """An eos token is kept and ends the loop (generate.rs:58-60); without
    eos ids the loop runs to max_new."""
    prompt = [int(t) for t in rng(7).integers(0, VOCAB, 5)]
    full = decoder(oracle, tiny).generate(prompt, 6)
    stop = full[2]
    first = full.index(stop)
    assert decoder(oracle, tiny).generate(prompt, 6, eos=(stop,)) == full[:first + 1]
    assert decoder(oracle, tiny).generate(prompt, 6, eos=()) == full


def test_argmax_total_last_maximum(oracle):
    x = np.array([0.5, 2.0, -1.0, 2.0, np.float32(-0.0), 1.0], np.float32)
    assert oracle.argmax_total(x) == 3  # equal maxima: max_by keeps the last
    assert oracle.argmax_total(np.array([np.nan, 1.0], np.float32)) == 0  # total_cmp puts NaN above +inf
    assert oracle.argmax_total(np.array([0.0, -0.0], np.float32)) == 0     # +0 > -0 under total_cmp


def test_bad_token(oracle, tiny):
    dec = decoder(oracle, tiny)
    with pytest.raises(oracle.OracleError):
        dec.forward(VOCAB, 0)
