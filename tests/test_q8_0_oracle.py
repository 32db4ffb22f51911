"""The Q8_0 mat-vec restatement in the oracle against the reference's own
tests for it (crates/llm-backend-cpu/tests/matvec.rs), with the same
fixtures (its LCG values and its Q8_0 weight quantizer) and bars."""
import numpy as np
import pytest


def test_quantize_uses_max_over_127_and_rounds_half_to_even(oracle):
    # tests/matvec.rs:39-48
    block = np.zeros(32, np.float32)
    block[0], block[1], block[2] = 127.0, 2.5, -3.5
    scales, quants = oracle.quantize_q8_0(block)
    assert scales.tolist() == [1.0]
    assert quants[:4].tolist() == [127, 2, -4, 0]


def test_matvec_equals_dot_of_dequantized_values(oracle):
    # tests/matvec.rs:50-66
    rows, cols = 64, 256
    w = oracle.q8_0_bytes_of(oracle.lcg_values(1, rows * cols))
    scales, quants = oracle.quantize_q8_0(oracle.lcg_values(2, cols))
    x_deq = (quants.reshape(-1, 32).astype(np.float32) * scales[:, None]).ravel()
    expected = oracle.dequant_q8_0(w).reshape(rows, cols).astype(np.float64) @ x_deq.astype(np.float64)
    actual = oracle.matvec_q8_0(w, rows, cols, scales, quants)
    assert np.max(np.abs(expected - actual)) < 1e-4


def test_fused_kernels_give_the_same_bits_as_separate_steps(oracle):
    # tests/matvec.rs:82-97, with the model's gelu_tanh (ops.rs:85-89) as the activation
    rows, cols = 300, 256
    gate = oracle.q8_0_bytes_of(oracle.lcg_values(5, rows * cols))
    up = oracle.q8_0_bytes_of(oracle.lcg_values(6, rows * cols))
    scales, quants = oracle.quantize_q8_0(oracle.lcg_values(7, cols))
    g = oracle.matvec_q8_0(gate, rows, cols, scales, quants)
    u = oracle.matvec_q8_0(up, rows, cols, scales, quants)
    separate = (oracle.gelu_tanh(g) * u).astype(np.float32)
    assert np.array_equal(oracle.geglu_q8_0(gate, up, rows, cols, scales, quants), separate)
    assert np.array_equal(oracle.matvec_q8_0_softcap(gate, rows, cols, scales, quants, 2.0), oracle.softcap(g, 2.0))


def test_matvec_is_close_to_the_f32_product(oracle):
    # tests/matvec.rs:99-110
    rows, cols = 64, 256
    w = oracle.lcg_values(1, rows * cols)
    x = oracle.lcg_values(2, cols)
    expected = w.reshape(rows, cols).astype(np.float64) @ x.astype(np.float64)
    scales, quants = oracle.quantize_q8_0(x)
    actual = oracle.matvec_q8_0(oracle.q8_0_bytes_of(w), rows, cols, scales, quants)
    assert np.max(np.abs(expected - actual)) < 0.25


def test_shape_errors(oracle):
    # tests/matvec.rs:131-134
    with pytest.raises(oracle.OracleError):
        oracle.quantize_q8_0(np.ones(31, np.float32))


def test_lcg_values_follow_the_reference_generator(oracle):
    # state' = state * 6364136223846793005 + 1 (mod 2^64); value = (state >> 40) / 2^23 - 1
    state, want = 3, []
    for _ in range(5):
        state = (state * 6364136223846793005 + 1) % (1 << 64)
        want.append(np.float32(state >> 40) / np.float32(1 << 23) - np.float32(1.0))
    assert np.array_equal(oracle.lcg_values(3, 5), np.array(want, np.float32))
