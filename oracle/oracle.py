"""ctypes binding of the CPU oracle (test infrastructure only).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
legs load this module, as the checker or the timed reference port. It is never
part of the product path.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liborc.so"

OK, CONTEXT_TOO_LONG, MISSING_LAYER, COMPUTE, NONFINITE, BAD_LAYER = 0, 1, 2, 4, 5, 6

_f32p = ctypes.POINTER(ctypes.c_float)


class HParams(ctypes.Structure):
    _fields_ = [
        ("n_layers", ctypes.c_int32), ("n_heads", ctypes.c_int32), ("n_kv_heads", ctypes.c_int32),
        ("head_dim_local", ctypes.c_int32), ("head_dim_global", ctypes.c_int32),
        ("sliding_window", ctypes.c_int32), ("shared_kv_layers", ctypes.c_int32),
        ("local_rope_base", ctypes.c_float), ("global_rope_base", ctypes.c_float),
        ("global_p", ctypes.c_float), ("rms_norm_eps", ctypes.c_float),
    ]


def build() -> Path:
    """Compile liborc.so with the committed Makefile (gcc only)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        sz = ctypes.c_size_t
        L.orc_rms_norm.argtypes = [_f32p, sz, _f32p, ctypes.c_float, _f32p]
        L.orc_dot_f32.argtypes = [_f32p, _f32p, sz]
        L.orc_dot_f32.restype = ctypes.c_float
        L.orc_softmax_f32.argtypes = [_f32p, sz, _f32p]
        L.orc_rope_neox.argtypes = [_f32p, sz, sz, ctypes.c_float, sz, _f32p, sz]
        L.orc_rope_sincos.argtypes = [sz, ctypes.c_float, sz, _f32p, _f32p, _f32p]
        L.orc_hparams_e2b.argtypes = [ctypes.POINTER(HParams)]
        L.orc_layer_is_global.argtypes = [ctypes.POINTER(HParams), ctypes.c_int32]
        L.orc_head_dim.argtypes = [ctypes.POINTER(HParams), ctypes.c_int32]
        L.orc_kv_source_layer.argtypes = [ctypes.POINTER(HParams), ctypes.c_int32,
                                          ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_int32)]
        L.orc_windowed_len.argtypes = [sz, sz, ctypes.POINTER(sz), ctypes.POINTER(sz)]
        L.orc_proportional_rope_freq_factors.argtypes = [sz, ctypes.c_float, _f32p]
        L.orc_attend.argtypes = [_f32p, _f32p, _f32p, sz, sz, sz, sz, ctypes.c_float, _f32p]
        L.orc_pool_init.argtypes = [ctypes.c_int]
        L.orc_kv_create.restype = ctypes.c_void_p
        L.orc_kv_destroy.argtypes = [ctypes.c_void_p]
        L.orc_kv_clear.argtypes = [ctypes.c_void_p]
        L.orc_kv_append.argtypes = [ctypes.c_void_p, sz, _f32p, _f32p, sz]
        L.orc_kv_append_rows.argtypes = [ctypes.c_void_p, sz, _f32p, _f32p, sz, sz]
        L.orc_kv_view.argtypes = [ctypes.c_void_p, sz, sz, ctypes.POINTER(_f32p), ctypes.POINTER(_f32p),
                                  ctypes.POINTER(sz), ctypes.POINTER(sz)]
        L.orc_attention_block.argtypes = [ctypes.c_void_p, ctypes.POINTER(HParams), ctypes.c_int32, sz,
                                          _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, ctypes.c_int, _f32p]
        L.orc_round_f16.argtypes = [ctypes.c_float]
        L.orc_round_f16.restype = ctypes.c_float
        L.orc_round_bf16.argtypes = [ctypes.c_float]
        L.orc_round_bf16.restype = ctypes.c_float
        L.orc_prefill_attend.argtypes = [_f32p, _f32p, _f32p, sz, sz, sz, sz, _f32p]
        u8p, i8p = ctypes.POINTER(ctypes.c_uint8), ctypes.POINTER(ctypes.c_int8)
        L.orc_quantize_q8_0.argtypes = [_f32p, sz, _f32p, i8p]
        L.orc_matvec_q8_0.argtypes = [u8p, sz, sz, _f32p, i8p, _f32p]
        L.orc_geglu_q8_0.argtypes = [u8p, u8p, sz, sz, _f32p, i8p, _f32p]
        L.orc_matvec_q8_0_softcap.argtypes = [u8p, sz, sz, _f32p, i8p, ctypes.c_float, _f32p]
        L.orc_gelu_tanh.argtypes = [ctypes.c_float]
        L.orc_gelu_tanh.restype = ctypes.c_float
        L.orc_softcap.argtypes = [ctypes.c_float, ctypes.c_float]
        L.orc_softcap.restype = ctypes.c_float
        L.orc_dequant_q8_0.argtypes = [u8p, sz, _f32p]
        L.orc_test_values.argtypes = [ctypes.c_uint64, sz, _f32p]
        L.orc_test_values.restype = None
        L.orc_test_q8_0_bytes.argtypes = [_f32p, sz, u8p]
        L.orc_test_q8_0_bytes.restype = None
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_f32p)


def f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


class OracleError(RuntimeError):
    def __init__(self, code: int, what: str):
        super().__init__(f"{what} failed with oracle status {code}")
        self.code = code


def _check(rc: int, what: str):
    if rc != OK:
        raise OracleError(rc, what)


def rms_norm(x, weight=None, eps=1e-6):
    x = f32(x)
    w = None if weight is None else f32(weight)
    if w is not None and w.size != x.size:
        raise OracleError(COMPUTE, "rms_norm")
    out = np.empty_like(x)
    _check(lib().orc_rms_norm(_p(x), x.size, _p(w), eps, _p(out)), "rms_norm")
    return out


def dot_f32(a, b) -> float:
    a, b = f32(a), f32(b)
    return float(lib().orc_dot_f32(_p(a), _p(b), a.size))


def softmax_f32(x):
    x = f32(x)
    out = np.empty_like(x)
    _check(lib().orc_softmax_f32(_p(x), x.size, _p(out)), "softmax_f32")
    return out


def rope_neox(x, position, base, n_rot, freq_factors=None):
    x = f32(x).copy()
    ff = None if freq_factors is None else f32(freq_factors)
    _check(lib().orc_rope_neox(_p(x), x.size, position, base, n_rot, _p(ff), 0 if ff is None else ff.size),
           "rope_neox")
    return x


def rope_sincos(position, base, n_rot, freq_factors=None):
    half = n_rot // 2
    s = np.empty(half, np.float32)
    c = np.empty(half, np.float32)
    ff = None if freq_factors is None else f32(freq_factors)
    lib().orc_rope_sincos(position, base, n_rot, _p(ff), _p(s), _p(c))
    return s, c


def hparams_e2b() -> HParams:
    hp = HParams()
    lib().orc_hparams_e2b(ctypes.byref(hp))
    return hp


def layer_is_global(hp: HParams, layer: int) -> bool:
    return bool(lib().orc_layer_is_global(ctypes.byref(hp), layer))


def head_dim(hp: HParams, layer: int) -> int:
    return int(lib().orc_head_dim(ctypes.byref(hp), layer))


def kv_source_layer(hp: HParams, layer: int):
    """Returns (source, None) or (None, detail) with detail 1/2/3 naming the
    KvShareError variant (LayerOutOfRange / TooManySharedLayers /
    NoEarlierLayerOfSameKind)."""
    src, det = ctypes.c_int32(-1), ctypes.c_int32(0)
    rc = lib().orc_kv_source_layer(ctypes.byref(hp), layer, ctypes.byref(src), ctypes.byref(det))
    return (src.value, None) if rc == OK else (None, det.value)


def windowed_len(seq_len, window):
    lo, hi = ctypes.c_size_t(), ctypes.c_size_t()
    lib().orc_windowed_len(seq_len, window, ctypes.byref(lo), ctypes.byref(hi))
    return lo.value, hi.value


def proportional_rope_freq_factors(head_dim_, p):
    out = np.empty(head_dim_ // 2, np.float32)
    lib().orc_proportional_rope_freq_factors(head_dim_, p, _p(out))
    return out


def attend(q, keys, values, n_heads, n_kv_heads, scale=1.0):
    q, keys, values = f32(q), f32(keys), f32(values)
    hd = q.size // n_heads
    length = keys.size // (n_kv_heads * hd) if keys.size else 0
    out = np.empty(q.size, np.float32)
    _check(lib().orc_attend(_p(q), _p(keys), _p(values), length, n_heads, n_kv_heads, hd, scale, _p(out)),
           "attend")
    return out


def pool_init(threads: int) -> int:
    return int(lib().orc_pool_init(threads))


def round_f16(a):
    return f32(a).astype(np.float16).astype(np.float32)


def round_bf16(a):
    a = f32(a)
    u = a.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def prefill_attend(q, k, v, n_heads, window):
    """q [T, n_heads, hd], k/v [T, hd] -> out [T, n_heads, hd]."""
    q, k, v = f32(q), f32(k), f32(v)
    T, hd = k.shape
    out = np.empty((T, n_heads, hd), np.float32)
    _check(lib().orc_prefill_attend(_p(q), _p(k), _p(v), T, n_heads, hd, window, _p(out)), "prefill_attend")
    return out


class KvCache:
    """context_memory.rs KvCache<Vec<f32>, Vec<f32>>: one row per position per layer."""

    def __init__(self):
        self.h = lib().orc_kv_create()

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_kv_destroy(self.h)
            self.h = None

    def clear(self):
        lib().orc_kv_clear(self.h)

    def append(self, layer, k, v):
        k, v = f32(k), f32(v)
        _check(lib().orc_kv_append(self.h, layer, _p(k), _p(v), k.size), "append")

    def append_rows(self, layer, k, v):
        k, v = f32(k), f32(v)
        _check(lib().orc_kv_append_rows(self.h, layer, _p(k), _p(v), k.shape[-1], k.shape[0]), "append_rows")

    def view(self, layer, length):
        kp, vp, w, m = _f32p(), _f32p(), ctypes.c_size_t(), ctypes.c_size_t()
        rc = lib().orc_kv_view(self.h, layer, length, ctypes.byref(kp), ctypes.byref(vp), ctypes.byref(w),
                               ctypes.byref(m))
        _check(rc, "view")
        if length == 0:
            return np.zeros((0, 0), np.float32), np.zeros((0, 0), np.float32)
        keys = np.ctypeslib.as_array(kp, shape=(length, w.value)).copy()
        values = np.ctypeslib.as_array(vp, shape=(length, w.value)).copy()
        return keys, values

    def attention_block(self, hp, layer, position, q_raw, k_raw, v_raw, q_norm_w, k_norm_w, rope_freqs,
                        kv_store=0):
        q_raw = f32(q_raw)
        k_raw = None if k_raw is None else f32(k_raw)
        v_raw = None if v_raw is None else f32(v_raw)
        out = np.empty(q_raw.size, np.float32)
        rc = lib().orc_attention_block(self.h, ctypes.byref(hp), layer, position, _p(q_raw), _p(k_raw),
                                       _p(v_raw), _p(f32(q_norm_w)), _p(None if k_norm_w is None else f32(k_norm_w)),
                                       _p(f32(rope_freqs)), kv_store, _p(out))
        _check(rc, "attention_block")
        return out


if __name__ == "__main__":  # pragma: no cover
    print(LIB_PATH, os.path.exists(LIB_PATH))


# ---------------------------------------------------------------------------
# Q8_0 mat-vec (crates/llm-backend-cpu/src/matvec.rs)
# ---------------------------------------------------------------------------

def _u8(a: np.ndarray):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8))


def _i8(a: np.ndarray):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_int8))


def quantize_q8_0(x):
    """(scales f32 [n/32], quants int8 [n]) as quantize_q8_0 (matvec.rs:36-54)."""
    x = f32(x).ravel()
    scales = np.empty(len(x) // 32, np.float32)
    quants = np.empty(len(x), np.int8)
    _check(lib().orc_quantize_q8_0(_p(x), len(x), _p(scales), _i8(quants)), "quantize_q8_0")
    return scales, quants


def _q8_call(fn, args, rows):
    out = np.empty(rows, np.float32)
    _check(fn(*args, _p(out)), fn.__name__)
    return out


def matvec_q8_0(w: np.ndarray, rows: int, cols: int, scales, quants):
    w = np.ascontiguousarray(w, np.uint8)
    return _q8_call(lib().orc_matvec_q8_0, (_u8(w), rows, cols, _p(scales), _i8(quants)), rows)


def geglu_q8_0(gate: np.ndarray, up: np.ndarray, rows: int, cols: int, scales, quants):
    gate, up = np.ascontiguousarray(gate, np.uint8), np.ascontiguousarray(up, np.uint8)
    return _q8_call(lib().orc_geglu_q8_0, (_u8(gate), _u8(up), rows, cols, _p(scales), _i8(quants)), rows)


def matvec_q8_0_softcap(w: np.ndarray, rows: int, cols: int, scales, quants, cap: float):
    w = np.ascontiguousarray(w, np.uint8)
    return _q8_call(lib().orc_matvec_q8_0_softcap, (_u8(w), rows, cols, _p(scales), _i8(quants), cap), rows)


def gelu_tanh(x):
    return np.array([lib().orc_gelu_tanh(float(v)) for v in np.ravel(x)], np.float32)


def softcap(x, cap: float):
    return np.array([lib().orc_softcap(float(v), cap) for v in np.ravel(x)], np.float32)


def dequant_q8_0(b: np.ndarray):
    b = np.ascontiguousarray(b, np.uint8)
    out = np.empty(len(b) // 34 * 32, np.float32)
    _check(lib().orc_dequant_q8_0(_u8(b), len(b), _p(out)), "dequant_q8_0")
    return out


def lcg_values(seed: int, n: int):
    """The reference test file's LCG values in [-1, 1) (tests/matvec.rs:10-18)."""
    out = np.empty(n, np.float32)
    lib().orc_test_values(seed, n, _p(out))
    return out


def q8_0_bytes_of(w):
    """The reference test file's Q8_0 quantizer for weights (tests/matvec.rs:21-31)."""
    w = f32(w).ravel()
    out = np.empty(len(w) // 32 * 34, np.uint8)
    lib().orc_test_q8_0_bytes(_p(w), len(w), _u8(out))
    return out


# ---------------------------------------------------------------------------
# E2B decoder, one token per call (crates/llm-gemma4/src/impl_/model.rs:252-449)
# ---------------------------------------------------------------------------

_u8p = ctypes.POINTER(ctypes.c_uint8)

_DEC_MATS = ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down", "inp_gate", "proj")
_DEC_NORMS = ("attn_norm", "attn_q_norm", "attn_k_norm", "post_attention_norm", "ffn_norm", "post_ffw_norm",
              "post_norm")


class DecLayerW(ctypes.Structure):
    _fields_ = [(n, _u8p) for n in _DEC_MATS] + [(n, _f32p) for n in _DEC_NORMS] + \
        [("layer_output_scale", ctypes.c_float)]


class DecW(ctypes.Structure):
    _fields_ = [("d_model", ctypes.c_int32), ("vocab", ctypes.c_int32), ("ple_dim", ctypes.c_int32),
                ("d_ff", ctypes.c_int32), ("final_logit_softcap", ctypes.c_float),
                ("token_embd", _u8p), ("ple_token_embd", _u8p), ("ple_model_proj", _u8p),
                ("ple_proj_norm", _f32p), ("output_norm", _f32p), ("rope_freqs", _f32p),
                ("layers", DecLayerW * 64)]


def _dec_bind():
    L = lib()
    if not getattr(L, "_dec_bound", False):
        L.orc_dec_forward.argtypes = [ctypes.c_void_p, ctypes.POINTER(HParams), ctypes.POINTER(DecW), ctypes.c_int32,
                                      ctypes.c_size_t, _f32p]
        L.orc_argmax_total.argtypes = [_f32p, ctypes.c_size_t]
        L.orc_argmax_total.restype = ctypes.c_int32
        L._dec_bound = True
    return L


def argmax_total(x) -> int:
    """sample.rs:27-36 at temperature 0: the last maximum under total_cmp."""
    x = f32(x).ravel()
    return int(_dec_bind().orc_argmax_total(_p(x), len(x)))


class Decoder:
    """Gemma4CpuModel's forward pass over host weights given by GGUF name
    (uint8 Q8_0 bytes for matrices, f32 for norms), with its own KvCache."""

    def __init__(self, hp: HParams, weights: dict, d_model: int, vocab: int, ple_dim: int, d_ff: int,
                 softcap: float, rope_freqs, layer_output_scales: dict):
        _dec_bind()
        own = HParams()  # the same fields, possibly from another binding's struct type
        for name, _ in HParams._fields_:
            setattr(own, name, getattr(hp, name))
        self.hp, self.vocab = own, vocab
        self._keep = []
        w = DecW()
        w.d_model, w.vocab, w.ple_dim, w.d_ff, w.final_logit_softcap = d_model, vocab, ple_dim, d_ff, softcap

        def u8(name):
            a = weights.get(name)
            if a is None:
                return None
            a = np.ascontiguousarray(a, np.uint8)
            self._keep.append(a)
            return a.ctypes.data_as(_u8p)

        def fl(name_or_array):
            a = weights.get(name_or_array) if isinstance(name_or_array, str) else name_or_array
            if a is None:
                return None
            a = f32(a)
            self._keep.append(a)
            return _p(a)

        w.token_embd = u8("token_embd.weight")
        w.ple_token_embd = u8("per_layer_token_embd.weight")
        w.ple_model_proj = u8("per_layer_model_proj.weight")
        w.ple_proj_norm = fl("per_layer_proj_norm.weight")
        w.output_norm = fl("output_norm.weight")
        w.rope_freqs = fl(np.asarray(rope_freqs, np.float32))
        for l in range(hp.n_layers):
            lw = w.layers[l]
            for n in _DEC_MATS:
                setattr(lw, n, u8(f"blk.{l}.{n}.weight"))
            for n in _DEC_NORMS:
                setattr(lw, n, fl(f"blk.{l}.{n}.weight"))
            lw.layer_output_scale = layer_output_scales.get(l, 1.0)
        self.w = w
        self.kv = KvCache()

    def clear(self):
        self.kv.clear()

    def forward(self, token: int, position: int) -> np.ndarray:
        logits = np.empty(self.vocab, np.float32)
        _check(lib().orc_dec_forward(self.kv.h, ctypes.byref(self.hp), ctypes.byref(self.w), token, position,
                                     _p(logits)), "dec_forward")
        return logits

    def generate(self, prompt, max_new: int, eos=()) -> list[int]:
        """generate_cpu (generate.rs:15-64) with greedy sampling; a token in
        `eos` (the model's eos_token_ids, model.rs:164) is kept and ends the
        generation (generate.rs:58-60)."""
        self.clear()
        logits = None
        for pos, tok in enumerate(prompt):
            logits = self.forward(int(tok), pos)
        out = []
        for index in range(max_new):
            out.append(argmax_total(logits))
            if out[-1] in eos:
                break
            if index + 1 == max_new:
                break
            logits = self.forward(out[-1], len(prompt) + len(out) - 1)
        return out
