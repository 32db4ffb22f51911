"""Python binding of libg4attn.so (the C ABI in include/g4attn.h).

Names follow the reference's attention boundary so that tests read like the
reference's own: `attend` (crates/llm-gemma4/src/impl_/model.rs:348),
`KvCache.append / view / clear` (crates/llm-eng/src/context_memory.rs:11-18),
`kv_source_layer`, `windowed_len`, `layer_is_global`, `head_dim`
(crates/llm-gemma4/src/{eng,idea}/mod.rs). Errors raise `EngError` carrying
the status code and the library's message.

Device memory is passed as torch CUDA tensors (only their data pointers cross
the boundary). There is no CPU fallback: every compute call goes to the CUDA
library, and importing this module fails if the library was not built.
"""
from __future__ import annotations

import atexit
import ctypes
import re
import weakref
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libg4attn.so"
HEADER = HERE.parent.parent / "include" / "g4attn.h"

OK, CONTEXT_TOO_LONG, MISSING_LAYER, MISSING_WEIGHT, COMPUTE, NONFINITE, BAD_LAYER, CUDA, NCCL, TIMEOUT, \
    OUT_OF_PAGES = range(11)
KV_F32, KV_F16 = 0, 1
K_DECODE_PREP, K_DECODE_MAIN, K_DECODE_COMBINE, K_DECODE_SPLITKV, K_PREFILL, K_MATVEC_Q8, K_CP_EXCHANGE, \
    K_CP_ATTEND_LOCAL, K_CP_ATTEND_REMOTE, K_CP_MERGE, K_COPY_IN, K_COPY_OUT, K_HOST_ISSUE, K_HOST_WAIT = range(14)
CP_KV_SHARDS, CP_GATHER_KV = 0, 1

_i32p = ctypes.POINTER(ctypes.c_int32)
_f32p = ctypes.POINTER(ctypes.c_float)
_vp = ctypes.c_void_p


class HParams(ctypes.Structure):
    _fields_ = [
        ("n_layers", ctypes.c_int32), ("n_heads", ctypes.c_int32), ("n_kv_heads", ctypes.c_int32),
        ("head_dim_local", ctypes.c_int32), ("head_dim_global", ctypes.c_int32),
        ("sliding_window", ctypes.c_int32), ("shared_kv_layers", ctypes.c_int32),
        ("local_rope_base", ctypes.c_float), ("global_rope_base", ctypes.c_float),
        ("global_p", ctypes.c_float), ("rms_norm_eps", ctypes.c_float),
    ]


class DecodeLayer(ctypes.Structure):
    _fields_ = [("layer", ctypes.c_int32), ("q_raw_dev", _vp), ("k_raw_dev", _vp), ("v_raw_dev", _vp),
                ("q_norm_w_dev", _vp), ("k_norm_w_dev", _vp), ("out_dev", _vp)]


class DecodeLayerHost(ctypes.Structure):
    _fields_ = [("layer", ctypes.c_int32), ("q_raw_host", _vp), ("k_raw_host", _vp), ("v_raw_host", _vp),
                ("q_norm_w_dev", _vp), ("k_norm_w_dev", _vp), ("out_host", _vp)]


class PrefillProblem(ctypes.Structure):
    _fields_ = [("head_dim", ctypes.c_int32), ("window", ctypes.c_int32), ("n_q", ctypes.c_int32),
                ("q_pos0", ctypes.c_int32), ("n_kv", ctypes.c_int32), ("kv_pos0", ctypes.c_int32),
                ("q_dev", _vp), ("k_dev", _vp), ("v_dev", _vp), ("out_dev", _vp), ("lse_dev", _vp)]


class CpProblem(ctypes.Structure):
    _fields_ = [("head_dim", ctypes.c_int32), ("seq_len", ctypes.c_int32), ("q_dev", _vp), ("k_dev", _vp),
                ("v_dev", _vp), ("out_dev", _vp)]


class EngError(RuntimeError):
    """A non-zero g4a_status (EngError of crates/llm-eng/src/error.rs)."""

    def __init__(self, code: int, message: str):
        super().__init__(f"[{code}] {message}")
        self.code = code
        self.message = message


def _load():
    if not LIB_PATH.exists():
        raise ImportError(f"{LIB_PATH} is missing: run `python gemma4-rs_b200/build.py` (no CPU fallback exists)")
    L = ctypes.CDLL(str(LIB_PATH))
    hp = ctypes.POINTER(HParams)
    L.g4a_hparams_e2b.argtypes = [hp]
    L.g4a_hparams_e2b.restype = None
    L.g4a_layer_is_global.argtypes = [hp, ctypes.c_int32]
    L.g4a_head_dim.argtypes = [hp, ctypes.c_int32]
    L.g4a_kv_source_layer.argtypes = [hp, ctypes.c_int32, _i32p, _i32p]
    L.g4a_windowed_len.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.POINTER(ctypes.c_int64),
                                   ctypes.POINTER(ctypes.c_int64)]
    L.g4a_windowed_len.restype = None
    L.g4a_proportional_rope_freq_factors.argtypes = [ctypes.c_int32, ctypes.c_float, _f32p]
    L.g4a_proportional_rope_freq_factors.restype = None
    L.g4a_ctx_create.argtypes = [ctypes.c_int, hp, _f32p, ctypes.c_int32, ctypes.POINTER(_vp)]
    L.g4a_ctx_destroy.argtypes = [_vp]
    L.g4a_ctx_destroy.restype = None
    L.g4a_last_error.argtypes = [_vp]
    L.g4a_last_error.restype = ctypes.c_char_p
    L.g4a_ctx_set_stream.argtypes = [_vp, _vp]
    L.g4a_sync.argtypes = [_vp]
    L.g4a_attend.argtypes = [_vp, _vp, _vp, _vp, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                             ctypes.c_float, _vp]
    L.g4a_kv_create.argtypes = [_vp, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                _i32p, ctypes.c_int32, ctypes.POINTER(_vp)]
    L.g4a_kv_destroy.argtypes = [_vp]
    L.g4a_kv_destroy.restype = None
    L.g4a_kv_clear.argtypes = [_vp, ctypes.c_int32]
    L.g4a_kv_len.argtypes = [_vp, ctypes.c_int32, ctypes.c_int32, ctypes.POINTER(ctypes.c_int64)]
    L.g4a_kv_append.argtypes = [_vp, ctypes.c_int32, ctypes.c_int32, _vp, _vp, ctypes.c_int64]
    L.g4a_kv_view.argtypes = [_vp, ctypes.c_int32, ctypes.c_int32, ctypes.c_int64, _vp, _vp]
    L.g4a_kv_append_tokens.argtypes = [_vp, ctypes.c_int32, ctypes.c_int32, _vp, _vp, _vp, ctypes.c_int64]
    L.g4a_decode.argtypes = [_vp, _vp, ctypes.c_int32, ctypes.POINTER(DecodeLayer), ctypes.c_int32, _i32p, _i32p]
    L.g4a_decode_host.argtypes = [_vp, _vp, ctypes.c_int32, ctypes.POINTER(DecodeLayerHost), ctypes.c_int32, _i32p,
                                  _i32p]
    L.g4a_decode_plan.argtypes = [_vp, _vp, ctypes.c_int32, ctypes.POINTER(DecodeLayer), ctypes.c_int32, _i32p,
                                  _i32p, ctypes.POINTER(_vp)]
    L.g4a_plan_run.argtypes = [_vp]
    L.g4a_plan_destroy.argtypes = [_vp]
    L.g4a_plan_destroy.restype = None
    L.g4a_prefill.argtypes = [_vp, ctypes.c_int32, ctypes.POINTER(PrefillProblem)]
    L.g4a_profile_enable.argtypes = [_vp, ctypes.c_int]
    L.g4a_profile_read.argtypes = [_vp, ctypes.c_int32, ctypes.POINTER(ctypes.c_double),
                                   ctypes.POINTER(ctypes.c_int64)]
    L.g4a_lse_merge.argtypes = [_vp, ctypes.c_int32, ctypes.POINTER(_vp), ctypes.POINTER(_vp), ctypes.c_int64,
                                ctypes.c_int32, ctypes.c_int32, _vp, _vp]
    L.g4a_matvec_q8_0.argtypes = [_vp, _vp, ctypes.c_int64, ctypes.c_int64, _vp, ctypes.c_int32, _vp]
    L.g4a_geglu_q8_0.argtypes = [_vp, _vp, _vp, ctypes.c_int64, ctypes.c_int64, _vp, ctypes.c_int32, _vp]
    L.g4a_matvec_q8_0_softcap.argtypes = [_vp, _vp, ctypes.c_int64, ctypes.c_int64, _vp, ctypes.c_int32,
                                          ctypes.c_float, _vp]
    L.g4a_quantize_q8_0.argtypes = [_vp, _vp, ctypes.c_int64, _vp, _vp]
    L.g4a_synth_q8_0.argtypes = [_vp, _vp, ctypes.c_int64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_float]
    L.g4a_synth_norm.argtypes = [_vp, _vp, ctypes.c_int64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_float,
                                 ctypes.c_float]
    L.g4a_model_create.argtypes = [_vp, _vp, ctypes.c_int32, ctypes.c_int32, ctypes.POINTER(_vp)]
    L.g4a_model_destroy.argtypes = [_vp]
    L.g4a_model_destroy.restype = None
    L.g4a_model_clear.argtypes = [_vp, ctypes.c_int32]
    L.g4a_model_len.argtypes = [_vp, ctypes.c_int32, _i32p]
    L.g4a_model_step.argtypes = [_vp, ctypes.c_int32, _i32p, _i32p, _i32p]
    L.g4a_model_prefill.argtypes = [_vp, ctypes.c_int32, _i32p, _i32p, ctypes.c_int32, _i32p]
    L.g4a_model_logits.argtypes = [_vp, ctypes.POINTER(_vp)]
    L.g4a_model_kv_view.argtypes = [_vp, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _vp, _vp]
    L.g4a_model_set_eos.argtypes = [_vp, _i32p, ctypes.c_int32]
    L.g4a_model_generate.argtypes = [_vp, ctypes.c_int32, _i32p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                     _i32p]
    L.g4a_debug_stall.argtypes = [_vp, ctypes.c_int32]
    L.g4a_cp_prefill.argtypes = [_vp, _vp, ctypes.c_int32, ctypes.POINTER(CpProblem)]
    L.g4a_cp_wait.argtypes = [_vp, _vp, ctypes.c_int32]
    L.g4a_nccl_unique_id.argtypes = [_vp]
    L.g4a_nccl_comm_init.argtypes = [ctypes.c_int32, ctypes.c_int32, _vp, ctypes.c_int, ctypes.POINTER(_vp)]
    L.g4a_nccl_comm_destroy.argtypes = [_vp]
    L.g4a_nccl_comm_destroy.restype = None
    return L


lib = _load()

# Handles still open when the interpreter exits are closed from an atexit hook,
# while the CUDA runtime is still up (finalizers that run later must not call
# into the library).
_live: "weakref.WeakSet" = weakref.WeakSet()
_exiting = False


def _close_all():
    global _exiting
    for obj in sorted(list(_live), key=lambda o: (isinstance(o, KvCache), isinstance(o, Context))):  # plans, caches, contexts
        try:
            obj.close()
        except Exception:
            pass
    _exiting = True


atexit.register(_close_all)


def declared_symbols() -> list[str]:
    """Every function the public header declares."""
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:[\w\s\*]+?)\b(g4a_\w+)\s*\(", text, re.M)))


# ---- hyperparameters and policies (host only) ----

def hparams_e2b() -> HParams:
    hp = HParams()
    lib.g4a_hparams_e2b(ctypes.byref(hp))
    return hp


def layer_is_global(hp: HParams, layer: int) -> bool:
    return bool(lib.g4a_layer_is_global(ctypes.byref(hp), layer))


def head_dim(hp: HParams, layer: int) -> int:
    return int(lib.g4a_head_dim(ctypes.byref(hp), layer))


def kv_source_layer(hp: HParams, layer: int):
    src, det = ctypes.c_int32(-1), ctypes.c_int32(0)
    rc = lib.g4a_kv_source_layer(ctypes.byref(hp), layer, ctypes.byref(src), ctypes.byref(det))
    return (src.value, None) if rc == OK else (None, det.value)


def windowed_len(seq_len: int, window: int):
    lo, hi = ctypes.c_int64(), ctypes.c_int64()
    lib.g4a_windowed_len(seq_len, window, ctypes.byref(lo), ctypes.byref(hi))
    return lo.value, hi.value


def proportional_rope_freq_factors(hd: int, p: float):
    out = (ctypes.c_float * (hd // 2))()
    lib.g4a_proportional_rope_freq_factors(hd, p, out)
    return list(out)


def _ptr(t) -> int | None:
    if t is None:
        return None
    assert t.is_cuda and t.is_contiguous(), "device tensors must be contiguous CUDA tensors"
    return t.data_ptr()


def _hptr(t) -> int | None:
    """Address of a contiguous float32 host buffer (numpy array or CPU tensor)."""
    if t is None:
        return None
    if isinstance(t, np.ndarray):
        assert t.dtype == np.float32 and t.flags["C_CONTIGUOUS"], "host buffers must be contiguous float32"
        return t.ctypes.data
    assert not t.is_cuda and t.is_contiguous(), "host buffers must be contiguous CPU tensors"
    return t.data_ptr()


class DecodeHostArgs:
    """A packed g4a_decode_host layer list (the buffers must stay alive)."""

    def __init__(self, layers: list[dict]):
        self.n = len(layers)
        self.arr = (DecodeLayerHost * max(1, self.n))()
        for i, a in enumerate(layers):
            self.arr[i] = DecodeLayerHost(a["layer"], _hptr(a["q_raw"]), _hptr(a.get("k_raw")),
                                          _hptr(a.get("v_raw")), _ptr(a.get("q_norm_w")), _ptr(a.get("k_norm_w")),
                                          _hptr(a["out"]))


class Context:
    """g4a_ctx: one device, one stream, RoPE tables and decode scratch."""

    def __init__(self, device: int = 0, hp: HParams | None = None, rope_freqs=None, max_positions: int = 4096):
        self.hp = hp or hparams_e2b()
        h = _vp()
        ff = None
        if rope_freqs is not None:
            arr = (ctypes.c_float * len(rope_freqs))(*[float(x) for x in rope_freqs])
            ff = ctypes.cast(arr, _f32p)
        rc = lib.g4a_ctx_create(device, ctypes.byref(self.hp), ff, max_positions, ctypes.byref(h))
        if rc != OK:
            raise EngError(rc, "g4a_ctx_create failed")
        self.h = h
        self.device = device
        _live.add(self)

    def close(self):
        if getattr(self, "h", None) and not _exiting:
            for o in [o for o in _live if not isinstance(o, Context) and getattr(o, "ctx", None) is self]:
                o.close()
            lib.g4a_ctx_destroy(self.h)
        self.h = None

    def __del__(self):
        self.close()

    def check(self, rc: int):
        if rc != OK:
            raise EngError(rc, lib.g4a_last_error(self.h).decode())

    def set_stream(self, stream_handle: int | None):
        self.check(lib.g4a_ctx_set_stream(self.h, stream_handle))

    def sync(self):
        self.check(lib.g4a_sync(self.h))

    def profile(self, enable: bool):
        self.check(lib.g4a_profile_enable(self.h, int(enable)))

    def debug_stall(self, kernel: int):
        """g4a_debug_stall: the next launch of `kernel` times out (tests)."""
        self.check(lib.g4a_debug_stall(self.h, kernel))

    def profile_read(self, kernel: int):
        """(total device ms, launches) of one kernel since profiling was enabled."""
        ms, n = ctypes.c_double(), ctypes.c_int64()
        self.check(lib.g4a_profile_read(self.h, kernel, ctypes.byref(ms), ctypes.byref(n)))
        return ms.value, n.value

    # model.rs:348 attend
    def attend(self, q, keys, values, n_heads: int, n_kv_heads: int, scale: float, out, length: int | None = None):
        hd = q.numel() // n_heads
        if length is None:
            length = keys.numel() // (n_kv_heads * hd) if keys is not None else 0
        self.check(lib.g4a_attend(self.h, _ptr(q), _ptr(keys) if length else None,
                                  _ptr(values) if length else None, length, n_heads, n_kv_heads, hd, scale,
                                  _ptr(out)))

    @staticmethod
    def _decode_args(layers, seq_ids, positions):
        arr = (DecodeLayer * max(1, len(layers)))()
        for i, a in enumerate(layers):
            arr[i] = DecodeLayer(a["layer"], _ptr(a["q_raw"]), _ptr(a.get("k_raw")), _ptr(a.get("v_raw")),
                                 _ptr(a.get("q_norm_w")), _ptr(a.get("k_norm_w")), _ptr(a["out"]))
        n = len(seq_ids)
        s = (ctypes.c_int32 * max(1, n))(*seq_ids)
        p = (ctypes.c_int32 * max(1, n))(*positions)
        return arr, n, s, p

    def decode(self, kv: "KvCache", layers: list[dict], seq_ids: list[int], positions: list[int]):
        arr, n, s, p = self._decode_args(layers, seq_ids, positions)
        self.check(lib.g4a_decode(self.h, kv.h, len(layers), arr, n, s, p))

    def decode_host(self, kv: "KvCache", layers, seq_ids, positions):
        """g4a_decode_host: q/k/v/out in host memory (dicts as decode(), with
        numpy arrays or CPU tensors, or a DecodeHostArgs); returns when the
        outputs are in the host buffers."""
        args = layers if isinstance(layers, DecodeHostArgs) else DecodeHostArgs(layers)
        s = np.ascontiguousarray(seq_ids, np.int32)
        p = np.ascontiguousarray(positions, np.int32)
        self.check(lib.g4a_decode_host(self.h, kv.h, args.n, args.arr, len(s), s.ctypes.data_as(_i32p),
                                       p.ctypes.data_as(_i32p)))

    def decode_plan(self, kv: "KvCache", layers: list[dict], seq_ids: list[int], positions: list[int]) -> "Plan":
        arr, n, s, p = self._decode_args(layers, seq_ids, positions)
        h = _vp()
        self.check(lib.g4a_decode_plan(self.h, kv.h, len(layers), arr, n, s, p, ctypes.byref(h)))
        return Plan(self, h)

    @staticmethod
    def prefill_args(problems: list[dict]) -> "PrefillArgs":
        """Packs a problem list once; pass the result to prefill() to skip the
        per-call packing (the tensors must stay alive)."""
        arr = (PrefillProblem * max(1, len(problems)))()
        for i, a in enumerate(problems):
            arr[i] = PrefillProblem(a["head_dim"], a.get("window", 0), a["n_q"], a.get("q_pos0", 0), a["n_kv"],
                                    a.get("kv_pos0", 0), _ptr(a["q"]), _ptr(a["k"]), _ptr(a["v"]), _ptr(a["out"]),
                                    _ptr(a.get("lse")))
        return PrefillArgs(arr, len(problems))

    def prefill(self, problems):
        """g4a_prefill over a list of problem dicts or a prefill_args() result."""
        args = problems if isinstance(problems, PrefillArgs) else self.prefill_args(problems)
        self.check(lib.g4a_prefill(self.h, args.n, args.arr))

    # ---- Q8_0 mat-vec (matvec.rs): w is a uint8 tensor of GGUF Q8_0 rows ----
    def matvec_q8_0(self, w, rows: int, cols: int, x, out, n_vec: int = 1):
        self.check(lib.g4a_matvec_q8_0(self.h, _ptr(w), rows, cols, _ptr(x), n_vec, _ptr(out)))

    def geglu_q8_0(self, gate, up, rows: int, cols: int, x, out, n_vec: int = 1):
        self.check(lib.g4a_geglu_q8_0(self.h, _ptr(gate), _ptr(up), rows, cols, _ptr(x), n_vec, _ptr(out)))

    def matvec_q8_0_softcap(self, w, rows: int, cols: int, x, cap: float, out, n_vec: int = 1):
        self.check(lib.g4a_matvec_q8_0_softcap(self.h, _ptr(w), rows, cols, _ptr(x), n_vec, cap, _ptr(out)))

    def quantize_q8_0(self, x, n: int, scales, quants):
        self.check(lib.g4a_quantize_q8_0(self.h, _ptr(x), n, _ptr(scales), _ptr(quants)))

    def lse_merge(self, outs, lses, rows: int, n_heads: int, hd: int, out, lse=None):
        n = len(outs)
        po = (_vp * n)(*[_ptr(t) for t in outs])
        pl = (_vp * n)(*[_ptr(t) for t in lses])
        self.check(lib.g4a_lse_merge(self.h, n, po, pl, rows, n_heads, hd, _ptr(out), _ptr(lse)))


    # ---- context-parallel prefill over an NCCL communicator ----
    def cp_prefill(self, comm: int, schedule: int, head_dim: int, seq_len: int, q, k, v, out):
        """g4a_cp_prefill: this rank's two zigzag chunks (q [2c, 8, hd], k/v
        [2c, hd] bf16, out [2c, 8, hd] f32) of a seq_len-token global layer;
        `comm` is an ncclComm_t as an integer (a torch ProcessGroupNCCL's
        _comm_ptr(), or NcclComm.ptr)."""
        pr = CpProblem(head_dim, seq_len, _ptr(q), _ptr(k), _ptr(v), _ptr(out))
        self.check(lib.g4a_cp_prefill(self.h, _vp(comm), schedule, ctypes.byref(pr)))

    def cp_wait(self, comm: int, timeout_ms: int):
        self.check(lib.g4a_cp_wait(self.h, _vp(comm), timeout_ms))


def nccl_unique_id() -> bytes:
    buf = (ctypes.c_uint8 * 128)()
    rc = lib.g4a_nccl_unique_id(buf)
    if rc != OK:
        raise EngError(rc, "nccl: no unique id (libnccl.so.2 missing?)")
    return bytes(buf)


class NcclComm:
    """A communicator made by the library (g4a_nccl_comm_init) for callers
    without one."""

    def __init__(self, n_ranks: int, rank: int, uid: bytes, device: int):
        buf = (ctypes.c_uint8 * 128)(*uid)
        h = _vp()
        rc = lib.g4a_nccl_comm_init(n_ranks, rank, buf, device, ctypes.byref(h))
        if rc != OK:
            raise EngError(rc, "nccl: communicator initialisation failed")
        self.h = h
        self.ptr = h.value
        _live.add(self)

    def close(self):
        if getattr(self, "h", None) and not _exiting:
            lib.g4a_nccl_comm_destroy(self.h)
        self.h = None

    def __del__(self):
        self.close()


class PrefillArgs:
    """A packed g4a_prefill problem array (see Context.prefill_args)."""

    def __init__(self, arr, n: int):
        self.arr = arr
        self.n = n


class Plan:
    """g4a_plan: a staged decode step that can be launched repeatedly."""

    def __init__(self, ctx: Context, h):
        self.ctx = ctx
        self.h = h
        _live.add(self)

    def run(self):
        self.ctx.check(lib.g4a_plan_run(self.h))

    def close(self):
        if getattr(self, "h", None) and not _exiting:
            lib.g4a_plan_destroy(self.h)
        self.h = None

    def __del__(self):
        self.close()


class KvCache:
    """g4a_kv: the paged device cache behind ContextMemory."""

    def __init__(self, ctx: Context, n_seqs: int, max_tokens: int, dtype: int = KV_F32, layers=None,
                 page_tokens: int = 64, n_pages: int = 0):
        self.ctx = ctx
        h = _vp()
        if layers is None:
            lp, nl = None, 0
        else:
            lp = (ctypes.c_int32 * max(1, len(layers)))(*layers)
            nl = len(layers)
        ctx.check(lib.g4a_kv_create(ctx.h, n_seqs, max_tokens, page_tokens, n_pages, dtype, lp, nl, ctypes.byref(h)))
        self.h = h
        self.dtype = dtype
        _live.add(self)

    def close(self):
        if getattr(self, "h", None) and not _exiting:
            lib.g4a_kv_destroy(self.h)
        self.h = None

    def __del__(self):
        self.close()

    def clear(self, seq: int = -1):
        self.ctx.check(lib.g4a_kv_clear(self.h, seq))

    def len(self, seq: int, layer: int) -> int:
        n = ctypes.c_int64()
        self.ctx.check(lib.g4a_kv_len(self.h, seq, layer, ctypes.byref(n)))
        return n.value

    def append(self, seq: int, layer: int, k, v):
        rows = k.shape[0] if k.dim() > 1 else 1
        self.ctx.check(lib.g4a_kv_append(self.h, seq, layer, _ptr(k), _ptr(v), rows))

    def append_tokens(self, seq: int, layer: int, k_raw, v_raw, k_norm_w):
        rows = k_raw.shape[0] if k_raw.dim() > 1 else 1
        self.ctx.check(lib.g4a_kv_append_tokens(self.h, seq, layer, _ptr(k_raw), _ptr(v_raw), _ptr(k_norm_w), rows))

    def view(self, seq: int, layer: int, length: int, keys_out, values_out):
        self.ctx.check(lib.g4a_kv_view(self.h, seq, layer, length, _ptr(keys_out), _ptr(values_out)))
