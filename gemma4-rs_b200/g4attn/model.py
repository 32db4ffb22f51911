"""The E2B decoder on the device (g4a_model_* of include/g4attn.h).

`synthetic_weights` fills device tensors, under the reference's GGUF tensor
names (crates/llm-gemma4/src/impl_/model.rs:27-42, 100-141), with seeded
random weights in the layout a GGUF file holds: Q8_0 bytes for every matrix
(values N(0, sigma) before quantization, d_ff = 2 * d_model as the
reference's synthetic model), f32 norm scales rounded to bf16 around 1.
`Model` is Gemma4CpuModel's forward pass and generate_cpu
(generate.rs:15-64) with greedy sampling, for many sequences at once.
"""
from __future__ import annotations

import ctypes
import sys

import numpy as np

from . import _i32p, _live, _vp, head_dim, kv_source_layer, lib, proportional_rope_freq_factors

Q8_BLOCK, Q8_BLOCK_BYTES = 32, 34
MAX_LAYERS = 64


class LayerWeights(ctypes.Structure):
    _fields_ = [(n, _vp) for n in ("attn_norm", "attn_q_norm", "attn_k_norm", "post_attention_norm", "ffn_norm",
                                   "post_ffw_norm", "post_norm", "attn_q", "attn_k", "attn_v", "attn_output",
                                   "ffn_gate", "ffn_up", "ffn_down", "inp_gate", "proj")] + \
        [("layer_output_scale", ctypes.c_float)]


class ModelWeights(ctypes.Structure):
    _fields_ = [("vocab_size", ctypes.c_int32), ("d_model", ctypes.c_int32), ("d_ff", ctypes.c_int32),
                ("ple_dim", ctypes.c_int32), ("final_logit_softcap", ctypes.c_float),
                ("token_embd", _vp), ("output_norm", _vp), ("ple_token_embd", _vp), ("ple_model_proj", _vp),
                ("ple_proj_norm", _vp), ("layers", LayerWeights * MAX_LAYERS)]


def blk(layer: int, name: str) -> str:
    """GGUF name of a per-layer weight (model.rs:40-42)."""
    return f"blk.{layer}.{name}.weight"


def fnv1a64(name: str) -> int:
    h = 0xCBF29CE484222325
    for b in name.encode():
        h = ((h ^ b) * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h


def q8_0_bytes(rows: int, cols: int) -> int:
    return rows * cols // Q8_BLOCK * Q8_BLOCK_BYTES


class Weights:
    """Device tensors by GGUF name; matrices as (uint8 Q8_0 bytes, (rows, cols))."""

    def __init__(self, hp, vocab: int, d_model: int, d_ff: int, ple_dim: int, softcap: float):
        self.hp, self.vocab, self.d_model, self.d_ff, self.ple_dim, self.softcap = hp, vocab, d_model, d_ff, ple_dim, \
            softcap
        self.tensors: dict = {}
        self.shapes: dict = {}
        self.scales: dict = {}  # layer_output_scale values

    def ptr(self, name: str):
        t = self.tensors.get(name)
        return None if t is None else t.data_ptr()

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.tensors.values())

    def struct(self) -> ModelWeights:
        s = ModelWeights()
        s.vocab_size, s.d_model, s.d_ff, s.ple_dim = self.vocab, self.d_model, self.d_ff, self.ple_dim
        s.final_logit_softcap = self.softcap
        s.token_embd, s.output_norm = self.ptr("token_embd.weight"), self.ptr("output_norm.weight")
        s.ple_token_embd = self.ptr("per_layer_token_embd.weight")
        s.ple_model_proj = self.ptr("per_layer_model_proj.weight")
        s.ple_proj_norm = self.ptr("per_layer_proj_norm.weight")
        for l in range(self.hp.n_layers):
            lw = s.layers[l]
            for f, _ in LayerWeights._fields_[:-1]:
                setattr(lw, f, self.ptr(blk(l, f)))
            lw.layer_output_scale = self.scales.get(l, 1.0)
        return s

    def host(self, name: str) -> np.ndarray:
        """A host copy (uint8 bytes of a matrix, f32 of a norm)."""
        return self.tensors[name].cpu().numpy()


def synthetic_weights(ctx, vocab: int = 262_144, d_model: int = 1536, d_ff: int | None = None, ple_dim: int = 256,
                      sigma: float = 0.02, seed: int = 0, softcap: float = 30.0) -> Weights:
    """Seeded random E2B weights on the context's device, GGUF names and layout."""
    import torch
    hp = ctx.hp
    d_ff = d_ff or 2 * d_model  # model.rs:106
    dev = torch.device("cuda", ctx.device)
    w = Weights(hp, vocab, d_model, d_ff, ple_dim, softcap)

    def q8(name, rows, cols):
        t = torch.empty(q8_0_bytes(rows, cols), dtype=torch.uint8, device=dev)
        ctx.check(lib.g4a_synth_q8_0(ctx.h, t.data_ptr(), rows * cols, seed, fnv1a64(name), sigma))
        w.tensors[name], w.shapes[name] = t, (rows, cols)

    def norm(name, n):
        t = torch.empty(n, dtype=torch.float32, device=dev)
        ctx.check(lib.g4a_synth_norm(ctx.h, t.data_ptr(), n, seed, fnv1a64(name), 1.0, 0.1))
        w.tensors[name], w.shapes[name] = t, (n,)

    q8("token_embd.weight", vocab, d_model)
    norm("output_norm.weight", d_model)
    width = hp.n_layers * ple_dim
    if ple_dim > 0:
        q8("per_layer_token_embd.weight", vocab, width)
        q8("per_layer_model_proj.weight", width, d_model)
        norm("per_layer_proj_norm.weight", ple_dim)
    scales = torch.empty(hp.n_layers, dtype=torch.float32, device=dev)
    ctx.check(lib.g4a_synth_norm(ctx.h, scales.data_ptr(), hp.n_layers, seed, fnv1a64("layer_output_scale"), 1.0,
                                 0.1))
    for l in range(hp.n_layers):
        hd = head_dim(hp, l)
        owner = kv_source_layer(hp, l)[0] == l
        for n in ("attn_norm", "post_attention_norm", "ffn_norm", "post_ffw_norm"):
            norm(blk(l, n), d_model)
        norm(blk(l, "attn_q_norm"), hd)
        q8(blk(l, "attn_q"), hp.n_heads * hd, d_model)
        if owner:  # shared-KV layers have no k/v projections that are used
            norm(blk(l, "attn_k_norm"), hd)
            q8(blk(l, "attn_k"), hp.n_kv_heads * hd, d_model)
            q8(blk(l, "attn_v"), hp.n_kv_heads * hd, d_model)
        q8(blk(l, "attn_output"), d_model, hp.n_heads * hd)
        q8(blk(l, "ffn_gate"), d_ff, d_model)
        q8(blk(l, "ffn_up"), d_ff, d_model)
        q8(blk(l, "ffn_down"), d_model, d_ff)
        if ple_dim > 0:
            q8(blk(l, "inp_gate"), ple_dim, d_model)
            q8(blk(l, "proj"), d_model, ple_dim)
            norm(blk(l, "post_norm"), d_model)
    ctx.sync()
    for l, v in enumerate(scales.cpu().tolist()):
        w.scales[l] = float(np.float32(v))
    return w


def rope_freqs(hp) -> np.ndarray:
    """rope_freqs.weight of the synthetic model (idea/mod.rs:158-165)."""
    return np.asarray(proportional_rope_freq_factors(hp.head_dim_global, hp.global_p), np.float32)


class Model:
    """g4a_model: the decoder over `weights` for up to max_seqs sequences."""

    def __init__(self, ctx, weights: Weights, max_seqs: int, max_tokens: int):
        self.ctx, self.weights = ctx, weights
        self._struct = weights.struct()
        h = _vp()
        ctx.check(lib.g4a_model_create(ctx.h, ctypes.byref(self._struct), max_seqs, max_tokens, ctypes.byref(h)))
        self.h = h
        self.max_seqs, self.max_tokens = max_seqs, max_tokens
        self._n = 0
        _live.add(self)

    def close(self):
        if getattr(self, "h", None) and not sys.modules[__package__]._exiting:
            lib.g4a_model_destroy(self.h)
        self.h = None

    def __del__(self):
        self.close()

    def clear(self, seq: int):
        self.ctx.check(lib.g4a_model_clear(self.h, seq))

    def len(self, seq: int) -> int:
        n = ctypes.c_int32()
        self.ctx.check(lib.g4a_model_len(self.h, seq, ctypes.byref(n)))
        return n.value

    def kv_view(self, seq: int, layer: int, length: int):
        """(keys, values) rows [0, length) of layer's K/V source, torch [length][hd]."""
        import torch
        src, _ = kv_source_layer(self.ctx.hp, layer)
        hd = head_dim(self.ctx.hp, src)
        k = torch.empty(length, hd, device=torch.device("cuda", self.ctx.device))
        v = torch.empty_like(k)
        self.ctx.check(lib.g4a_model_kv_view(self.h, seq, layer, length, k.data_ptr(), v.data_ptr()))
        self.ctx.sync()
        return k, v

    def step(self, seq_ids, tokens) -> list[int]:
        """One token per sequence; returns the greedy next tokens."""
        n = len(seq_ids)
        ids = (ctypes.c_int32 * n)(*seq_ids)
        tok = (ctypes.c_int32 * n)(*tokens)
        nxt = (ctypes.c_int32 * n)()
        self.ctx.check(lib.g4a_model_step(self.h, n, ids, tok, nxt))
        self._n = n
        return list(nxt)

    def prefill(self, seq_ids, tokens) -> list[int]:
        """A prompt per sequence, tokens [n][len], appended at each sequence's
        length in chunks of many positions; returns the greedy token after
        each prompt (logits() then gives those n rows)."""
        tokens = np.ascontiguousarray(tokens, np.int32)
        n, length = tokens.shape
        if len(seq_ids) != n:
            raise ValueError("one prompt per sequence id")
        ids = (ctypes.c_int32 * n)(*seq_ids)
        nxt = (ctypes.c_int32 * n)()
        self.ctx.check(lib.g4a_model_prefill(self.h, n, ids, tokens.ctypes.data_as(_i32p), length, nxt))
        self._n = n
        return list(nxt)

    def logits(self):
        """A copy of the last step's soft-capped logits, torch [n][vocab] on the device."""
        import torch
        p = _vp()
        self.ctx.check(lib.g4a_model_logits(self.h, ctypes.byref(p)))

        class _View:
            __cuda_array_interface__ = {"shape": (self._n, self.weights.vocab), "typestr": "<f4",
                                        "data": (p.value, False), "version": 3, "strides": None}
        return torch.as_tensor(_View(), device=torch.device("cuda", self.ctx.device)).clone()

    def set_eos(self, ids) -> None:
        """eos_token_ids: generate() ends a sequence after emitting one."""
        arr = (ctypes.c_int32 * max(1, len(ids)))(*ids)
        self.ctx.check(lib.g4a_model_set_eos(self.h, arr, len(ids)))

    def generate(self, prompts, max_new: int, max_context: int | None = None) -> np.ndarray:
        """generate_cpu with greedy sampling for rows 0..n-1: [n][max_new]
        tokens (-1 after a sequence's eos token)."""
        prompts = np.ascontiguousarray(prompts, np.int32)
        n, plen = prompts.shape
        out = np.zeros((n, max_new), np.int32)
        mc = self.max_tokens if max_context is None else max_context
        self.ctx.check(lib.g4a_model_generate(self.h, n, prompts.ctypes.data_as(_i32p), plen, max_new, mc,
                                              out.ctypes.data_as(_i32p)))
        return out
