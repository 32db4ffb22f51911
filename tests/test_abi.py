"""The C-ABI library loads, exports every symbol the header declares, and its
host-only policy functions agree with the oracle (no GPU needed)."""
import ctypes

import numpy as np


def test_library_exports_every_declared_symbol():
    import g4attn
    names = g4attn.declared_symbols()
    assert len(names) >= 20
    for n in names:
        assert hasattr(g4attn.lib, n), n
        assert ctypes.cast(getattr(g4attn.lib, n), ctypes.c_void_p).value


def test_header_declares_the_boundary():
    import g4attn
    names = set(g4attn.declared_symbols())
    for n in ("g4a_attend", "g4a_decode", "g4a_prefill", "g4a_kv_append", "g4a_kv_view", "g4a_kv_clear",
              "g4a_kv_source_layer", "g4a_windowed_len", "g4a_lse_merge", "g4a_sync"):
        assert n in names


def test_policies_match_oracle(oracle):
    import g4attn
    hp, ohp = g4attn.hparams_e2b(), oracle.hparams_e2b()
    for f in ("n_layers", "n_heads", "n_kv_heads", "head_dim_local", "head_dim_global", "sliding_window",
              "shared_kv_layers", "local_rope_base", "global_rope_base", "global_p", "rms_norm_eps"):
        assert getattr(hp, f) == getattr(ohp, f), f
    for layer in range(-1, 37):
        assert g4attn.kv_source_layer(hp, layer) == oracle.kv_source_layer(ohp, layer)
        if 0 <= layer < 35:
            assert g4attn.layer_is_global(hp, layer) == oracle.layer_is_global(ohp, layer)
            assert g4attn.head_dim(hp, layer) == oracle.head_dim(ohp, layer)
    for n in (0, 1, 511, 512, 513, 628, 1000, 4096):
        assert g4attn.windowed_len(n, 512) == oracle.windowed_len(n, 512)
    assert np.array_equal(np.array(g4attn.proportional_rope_freq_factors(512, 0.25), np.float32),
                          oracle.proportional_rope_freq_factors(512, 0.25))


def test_kv_source_errors_match_reference():
    """layer_pattern.rs:69-86 through the C ABI."""
    import g4attn
    hp = g4attn.hparams_e2b()
    assert g4attn.kv_source_layer(hp, 35) == (None, 1)
    hp.shared_kv_layers = 35
    assert g4attn.kv_source_layer(hp, 0) == (None, 2)
    hp = g4attn.hparams_e2b()
    hp.shared_kv_layers = 31
    assert g4attn.kv_source_layer(hp, 34) == (None, 3)


def test_no_context_without_device():
    """Without a usable device the context fails loudly (no CPU fallback)."""
    import pytest
    import torch
    import g4attn
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(g4attn.EngError):
        g4attn.Context(0)
