"""GPU: dequantization and layout parity through the C ABI (bit-exact)."""
from pathlib import Path

import numpy as np
import pytest
import torch

from tests.test_oracle import GEO, TYPES, load_golden, same_bits

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", list(TYPES))
def test_dequant_matches_gguf_golden(backend, name):
    t = TYPES[name]
    blocks, exp, _ = load_golden(name)
    elems, nbytes = GEO[t]
    nb = blocks.size // nbytes
    w = backend.upload_quant(t, blocks, nb, elems)  # one block per row, 58 rows (ragged tile)
    got = backend.dequant(w.quant).cpu().numpy().reshape(-1)
    assert same_bits(got, exp)
    # layout round trip: TILED16 -> GGUF gives back the uploaded bytes
    assert np.array_equal(w.quant.to_gguf(), blocks)


@pytest.mark.parametrize("t", [12, 14, 8])
@pytest.mark.parametrize("n,k", [(1, 256), (37, 1024), (64, 512)])
def test_dequant_matches_oracle(backend, oracle, t, n, k):
    from ocelotl_b200 import synth
    blocks = synth.quant_blocks(t, n, k, 11, f"dq{t}")
    w = backend.upload_quant(t, blocks, n, k)
    got = backend.dequant(w.quant).cpu().numpy()
    ref = oracle.dequant(t, blocks.numpy(), n, k)
    assert same_bits(got, ref)
    assert np.array_equal(w.quant.to_gguf(), blocks.numpy())
    # QuantBuffer.to_host is the dequantized f32 (DeviceBuffer::to_host contract)
    assert w.len_f32() == n * k
    assert same_bits(w.to_host_owned(), ref.reshape(-1))


@pytest.mark.parametrize("t", [12, 14, 8])
def test_upload_from_device_equals_host_upload(backend, t):
    from ocelotl_b200 import synth
    n, k = 48, 768
    blocks = synth.quant_blocks(t, n, k, 5, "dev")
    a = backend.upload_quant(t, blocks, n, k)
    b = backend.upload_quant(t, blocks.cuda(), n, k)
    assert torch.equal(backend.dequant(a.quant), backend.dequant(b.quant))


def test_embed_rows_q8_0(backend, oracle):
    from ocelotl_b200 import synth
    n, k = 300, 4096
    blocks = synth.quant_blocks(8, n, k, 9, "emb")
    table = backend.upload_quant(8, blocks, n, k)
    ids = torch.tensor([0, 17, 299, 5, 17], dtype=torch.int32, device="cuda")
    got = backend.embed_rows(table, ids).cpu().numpy()
    ref = oracle.dequant(8, blocks.numpy(), n, k)[ids.cpu().numpy()]
    assert same_bits(got, ref)
    assert backend.take_bad_ids() == 0
    bad = torch.tensor([3, -1, 300], dtype=torch.int32, device="cuda")
    got = backend.embed_rows(table, bad).cpu().numpy()
    assert backend.take_bad_ids() == 2
    assert same_bits(got[0], oracle.dequant(8, blocks.numpy(), n, k)[3])
    assert not got[1:].any()
