"""CPU oracle checks: golden dequant vectors and the reference's multiply properties.

Mirrors the reference's own linear tests (crates/kernels/src/lib.rs):
hand-computed cases (:2650-2735), tile tails bit-exact vs a naive loop
(:2843-2889), threaded == serial bit-for-bit (:2891-2942), AVX2 within 1e-4 of
scalar with odd K=200 / N=33 tails (:2944-3003).
"""
import hashlib
import struct
from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"
TYPES = {"q4_k": 12, "q6_k": 14, "q8_0": 8}
GEO = {12: (256, 144), 14: (256, 210), 8: (32, 34)}


def load_golden(name):
    z = np.load(GOLDEN / f"dequant_{name}.npz")
    return z["blocks"], z["expected"], str(z["sha256"])


def same_bits(a, b):
    """Bit-exact, with any NaN matching any NaN (payload quieting differs across ISAs)."""
    a = np.asarray(a, dtype=np.float32)
    b = np.asarray(b, dtype=np.float32)
    na, nb = np.isnan(a), np.isnan(b)
    return bool(np.array_equal(na, nb) and np.array_equal(a[~na].view(np.uint32), b[~nb].view(np.uint32)))


@pytest.mark.parametrize("name", list(TYPES))
def test_golden_digest_is_self_consistent(name):
    _, exp, digest = load_golden(name)
    assert hashlib.sha256(exp.tobytes()).hexdigest() == digest


@pytest.mark.parametrize("name", list(TYPES))
def test_oracle_dequant_matches_gguf_golden(oracle, name):
    t = TYPES[name]
    blocks, exp, _ = load_golden(name)
    elems, nbytes = GEO[t]
    nb = blocks.size // nbytes
    got = oracle.dequant(t, blocks, nb, elems)  # one block per row
    assert same_bits(got.reshape(-1), exp)


def test_oracle_dequant_rows_of_many_blocks(oracle):
    # the same golden blocks seen as [rows, k] with several blocks per row
    blocks, exp, _ = load_golden("q4_k")
    got = oracle.dequant(12, blocks[: 48 * 144], 12, 4 * 256)
    assert same_bits(got.reshape(-1), exp[: 48 * 256])


def test_f16_decode_matches_ieee_for_all_bit_patterns(oracle):
    # crates/loader/src/safetensors_values.rs:155-183 is the exact IEEE conversion
    for h in list(range(0, 0x10000, 97)) + [0x0001, 0x03FF, 0x0400, 0x7BFF, 0x7C00, 0xFC00, 0x8001]:
        ref = np.array([h], dtype=np.uint16).view(np.float16).astype(np.float32)[0]
        got = np.float32(oracle.f16_to_f32(h))
        if np.isnan(ref):
            assert np.isnan(got)
        else:
            assert struct.pack("<f", got) == struct.pack("<f", ref), hex(h)


def test_linear_hand_computed(oracle):
    # out[r,o] = b[o] + sum_k x[r,k] w[o,k]
    x = np.array([1, 2, 3, 4, 5, 6], np.float32)          # 2 x 3
    w = np.array([7, 9, 11, 8, 10, 12], np.float32)         # 2 x 3 (out x in)
    out = oracle.linear_out_by_in(x, 2, 3, w, 2)
    assert out.reshape(-1).tolist() == [58, 64, 139, 154]
    out = oracle.linear_out_by_in(x, 2, 3, w, 2, bias=np.array([1, -1], np.float32))
    assert out.reshape(-1).tolist() == [59, 63, 140, 153]


def _closed_form(n, a, b):
    i = np.arange(n, dtype=np.float64)
    return np.sin(i * a + b).astype(np.float32)


def test_linear_sequential_k_bits(oracle):
    # bit-exact vs a naive sequential-k f32 loop (tile tails: rows=6, out=7)
    rows, k, n = 6, 37, 7
    x = _closed_form(rows * k, 0.013, 0.1)
    w = np.cos(np.arange(n * k) * 0.019).astype(np.float32)
    b = _closed_form(n, 0.5, 0.2)
    out = oracle.linear_out_by_in(x, rows, k, w, n, bias=b)
    ref = np.empty((rows, n), np.float32)
    for r in range(rows):
        for o in range(n):
            acc = np.float32(b[o])
            for i in range(k):
                acc = np.float32(acc + np.float32(x[r * k + i] * w[o * k + i]))
            ref[r, o] = acc
    assert np.array_equal(out.view(np.uint32), ref.view(np.uint32))


def test_avx2_close_to_scalar_with_tails(oracle):
    if not oracle.lib().orc_has_avx2():
        pytest.skip("host lacks avx2+fma")
    rows, k, n = 9, 200, 33
    x = _closed_form(rows * k, 0.013, 0.0)
    w = np.cos(np.arange(n * k) * 0.019).astype(np.float32)
    b = _closed_form(n, 0.3, 0.0)
    s = oracle.linear_out_by_in(x, rows, k, w, n, bias=b)
    a = oracle.linear_out_by_in(x, rows, k, w, n, bias=b, avx2=True)
    assert np.allclose(a, s, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("t", [12, 14, 8])
def test_q_linear_equals_dequant_then_linear_bitwise(oracle, t):
    import torch
    from ocelotl_b200 import synth
    n, k, rows = 21, 512, 3
    blocks = synth.quant_blocks(t, n, k, 7, f"w{t}").numpy()
    x = synth.activations(rows, k, 7, "x").numpy()
    bias = synth.activations(1, n, 7, "b").numpy().reshape(-1)
    w = oracle.dequant(t, blocks, n, k)
    ref = oracle.linear_out_by_in(x, rows, k, w, n, bias=bias)
    got = oracle.q_linear(t, blocks, x, rows, k, n, bias=bias)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    # row-chunk threading is bit-identical to serial
    got4 = oracle.q_linear(t, blocks, x, rows, k, n, bias=bias, threads=4)
    assert np.array_equal(got4.view(np.uint32), ref.view(np.uint32))
    del torch


def test_q_linear_avx2_threaded_bitwise(oracle):
    if not oracle.lib().orc_has_avx2():
        pytest.skip("host lacks avx2+fma")
    from ocelotl_b200 import synth
    n, k, rows = 37, 256, 8
    blocks = synth.quant_blocks(12, n, k, 3, "w").numpy()
    x = synth.activations(rows, k, 3, "x").numpy()
    w = oracle.dequant(12, blocks, n, k)
    ref = oracle.linear_out_by_in(x, rows, k, w, n, avx2=True)
    a1 = oracle.q_linear(12, blocks, x, rows, k, n, avx2=True)
    a3 = oracle.q_linear(12, blocks, x, rows, k, n, avx2=True, threads=3)
    assert np.array_equal(a1.view(np.uint32), ref.view(np.uint32))
    assert np.array_equal(a3.view(np.uint32), ref.view(np.uint32))


def test_oracle_rejects_bad_k(oracle):
    with pytest.raises(ValueError):
        oracle.dequant(12, np.zeros(144, np.uint8), 1, 100)


def test_silu_hand_checked_values(oracle):
    # silu(z) = z / (1 + e^-z): 0 -> 0, 1 -> 0.73105858, -1 -> -0.26894143, 2 -> 1.76159416, 3 -> 2.85772238
    v = oracle.silu_inplace(np.array([0.0, 1.0, -1.0, 2.0, 3.0], np.float32))
    assert np.allclose(v, [0.0, 0.73105858, -0.26894143, 1.76159416, 2.85772238], atol=1e-6)
    # large negative: sigmoid underflows to 0, silu -> 0 (no NaN)
    big = oracle.silu_inplace(np.array([-200.0, -1e30, 200.0], np.float32))
    assert big[0] == 0 and big[1] == 0 and big[2] == 200.0


def test_oracle_mlp_doc_example(oracle):
    from tests.mlp_cases import doc_example
    x, gate, up, down, hidden, inter = doc_example()
    act, out = oracle.q_mlp_gated_silu(8, gate, up, 8, down, x, 1, hidden, inter)
    assert np.allclose(act, 3.5231884, atol=1e-5)
    assert np.allclose(out, 3.5231884, atol=1e-5)


def test_greedy_sample_reference_cases(oracle):
    # peak at 3; three-way tie at 1, 2, 3 -> lowest id
    assert oracle.greedy_sample([0.1, 0.5, 0.3, 0.9, 0.2]) == 3
    assert oracle.greedy_sample([0.1, 0.5, 0.5, 0.5, 0.2]) == 1
    assert oracle.greedy_sample([7.0]) == 0
    with pytest.raises(ValueError):
        oracle.greedy_sample([])
    nan = float("nan")
    assert oracle.greedy_sample([nan, 5.0, 9.0]) == 0        # NaN at 0 is never displaced
    assert oracle.greedy_sample([1.0, nan, 0.5, nan]) == 0   # NaN never wins
    assert oracle.greedy_sample([-0.0, 0.0]) == 0            # -0.0 == +0.0
    assert oracle.greedy_sample([-np.inf, -np.inf]) == 0
    assert oracle.greedy_sample([1.0, np.inf, np.inf]) == 1


def test_greedy_sample_fast_matches_scan(oracle):
    rng = np.random.default_rng(5)
    for trial in range(300):
        n = int(rng.integers(1, 40))
        v = rng.integers(-3, 4, size=n).astype(np.float32)   # many ties
        mask = rng.random(n) < 0.15
        v[mask] = np.nan
        if rng.random() < 0.2:
            v[rng.integers(0, n)] = -0.0
        assert oracle.greedy_sample_fast(v) == oracle.greedy_sample(v), v
