"""GPU: greedy sampling (argmax over logits) vs the reference scan, bit-exact ids
(crates/runtime/src/sampling.rs:29-52)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_reference_cases(backend):
    nan = float("nan")
    cases = [[0.1, 0.5, 0.3, 0.9, 0.2], [0.1, 0.5, 0.5, 0.5, 0.2], [7.0], [nan, 5.0, 9.0], [1.0, nan, 0.5, nan],
             [-0.0, 0.0], [-np.inf, -np.inf], [1.0, np.inf, np.inf]]
    want = [3, 1, 0, 0, 0, 0, 0, 1]
    for c, w in zip(cases, want):
        assert backend.greedy_sample(np.array(c, np.float32)) == w, c


def test_empty_is_an_error(backend):
    from ocelotl_b200.errors import KernelError
    with pytest.raises(KernelError):
        backend.greedy_sample(np.zeros(0, np.float32))


@pytest.mark.parametrize("vocab", [1, 5, 4095, 4096, 4097, 32000, 128256, 151936])
def test_random_rows_with_ties_and_nans(backend, oracle, vocab):
    rng = np.random.default_rng(vocab)
    rows = 7
    v = rng.integers(-50, 51, size=(rows, vocab)).astype(np.float32)  # dense ties
    v[rng.random((rows, vocab)) < 0.01] = np.nan
    v[1, 0] = np.nan                                                   # NaN at index 0
    v[2, rng.integers(0, vocab)] = np.inf
    v[3] = -0.0
    v[3, vocab // 2] = 0.0
    logits = torch.from_numpy(v).cuda()
    ids = backend.greedy_sample(logits).cpu().numpy()
    want = [oracle.greedy_sample_fast(v[r]) for r in range(rows)]
    assert list(ids) == want
    # a second launch (slots and counters were reset by the first)
    ids2 = backend.greedy_sample(logits).cpu().numpy()
    assert list(ids2) == want


def test_unaligned_rows(backend, oracle):
    rng = np.random.default_rng(1)
    vocab, rows = 1001, 5  # row starts not 16-byte aligned
    v = rng.standard_normal((rows, vocab)).astype(np.float32)
    ids = backend.greedy_sample(torch.from_numpy(v).cuda()).cpu().numpy()
    assert list(ids) == [oracle.greedy_sample_fast(v[r]) for r in range(rows)]


def test_head_gemv_then_argmax(backend, oracle):
    """Output head: Q6_K vocab GEMV (f32 logits) then greedy sampling on the device."""
    from ocelotl_b200 import synth
    vocab, k = 4000, 512
    blocks = synth.quant_blocks(14, vocab, k, 3, "head")
    w = backend.upload_quant(14, blocks, vocab, k)
    x = synth.activations(2, k, 3, "x")
    logits = torch.empty(2, vocab, device="cuda")
    backend.linear_dev(w, x.cuda(), 2, logits)
    ids = backend.greedy_sample(logits).cpu().numpy()
    ref_logits = oracle.q_linear(14, blocks.numpy(), x.numpy(), 2, k, vocab)
    got_l = logits.cpu().numpy()
    assert list(ids) == [oracle.greedy_sample_fast(got_l[r]) for r in range(2)]
    # the device logits agree with the oracle's to GEMV tolerance, so the ids
    # agree unless the top two logits are closer than that
    for r in range(2):
        top2 = np.sort(ref_logits[r])[-2:]
        if top2[1] - top2[0] > 1e-3 * abs(top2[1]) + 1e-3:
            assert ids[r] == oracle.greedy_sample(ref_logits[r])
