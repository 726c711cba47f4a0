"""GPU: weights loaded from a GGUF file run through the quantized linear path."""
import numpy as np
import pytest

from tests.gguf_writer import write_gguf
from tests.test_oracle import same_bits
from tests.tolerance import GEMV_RTOL, rel_err

pytestmark = pytest.mark.gpu


def test_gguf_file_to_gemv(backend, oracle, tmp_path):
    from ocelotl_b200 import gguf, synth
    n, k = 96, 1024
    q4 = synth.quant_blocks(12, n, k, 2, "file.q4").numpy()
    q6 = synth.quant_blocks(14, n, k, 2, "file.q6").numpy()
    p = tmp_path / "w.gguf"
    write_gguf(p, [("a.weight", [k, n], 12, q4.tobytes()), ("b.weight", [k, n], 14, q6.tobytes())])
    m = gguf.inspect(p)
    x = synth.activations(2, k, 2, "file.x").numpy()
    for name, t, blk in (("a.weight", 12, q4), ("b.weight", 14, q6)):
        w = gguf.upload_quant_tensor(backend, m, name)
        assert np.array_equal(w.quant.to_gguf(), blk)
        assert same_bits(backend.dequant(w.quant).cpu().numpy(), oracle.dequant(t, blk, n, k))
        out = np.zeros(2 * n, np.float32)
        backend.linear_out_by_in(x, 2, k, w, n, None, out)
        assert rel_err(out.reshape(2, n), oracle.q_linear(t, blk, x, 2, k, n)) <= GEMV_RTOL
