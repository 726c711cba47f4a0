"""CPU: GGUF reader (header walk as inspect_gguf, crates/loader/src/gguf_inspect.rs:224-414,
plus quantized payload sizing and access)."""
import numpy as np
import pytest

from ocelotl_b200 import UnsupportedError, gguf, synth
from ocelotl_b200.ggml import byte_len
from tests.gguf_writer import write_gguf


def blocks(t, n, k, seed=0):
    return synth.quant_blocks(t, n, k, seed, f"gg{t}").numpy()


def test_reads_quantized_tensors_and_metadata(tmp_path):
    q4 = blocks(12, 8, 512)
    q6 = blocks(14, 4, 256)
    q8 = blocks(8, 3, 64)
    f32 = np.arange(6, dtype=np.float32)
    p = tmp_path / "m.gguf"
    write_gguf(p, [("blk.0.ffn_gate.weight", [512, 8], 12, q4.tobytes()),
                   ("blk.0.ffn_down.weight", [256, 4], 14, q6.tobytes()),
                   ("token_embd.weight", [64, 3], 8, q8.tobytes()),
                   ("norm.weight", [6], 0, f32.tobytes())],
               metadata={"general.architecture": ("str", "llama"), "x.scales": ("f32arr", [1.0, 2.5])},
               alignment=64)
    m = gguf.inspect(p)
    assert m.version == 3 and m.alignment == 64 and m.data_start % 64 == 0
    assert m.metadata["general.architecture"] == "llama" and m.metadata["x.scales"] == [1.0, 2.5]
    t = m.tensor("blk.0.ffn_gate.weight")
    assert (t.k, t.n_rows, t.byte_len) == (512, 8, byte_len(12, 8, 512))
    assert np.array_equal(gguf.read_payload(m, "blk.0.ffn_gate.weight"), q4)
    assert np.array_equal(gguf.read_payload(m, "blk.0.ffn_down.weight"), q6)
    assert np.array_equal(gguf.read_payload(m, "token_embd.weight"), q8)
    assert np.array_equal(gguf.read_payload(m, "norm.weight").view(np.float32), f32)


def test_quant_byte_len_matches_block_geometry():
    assert gguf.tensor_byte_len(12, [4096, 14336]) == 14336 * 16 * 144
    assert gguf.tensor_byte_len(14, [14336, 4096]) == 4096 * 56 * 210
    assert gguf.tensor_byte_len(8, [4096, 128256]) == 128256 * 128 * 34
    assert gguf.tensor_byte_len(12, [100, 2]) is None  # not whole blocks
    assert gguf.tensor_byte_len(2, [32, 2]) is None    # Q4_0: not sized by this path


@pytest.mark.parametrize("kw,exc,needle", [
    ({"magic": b"GGUX"}, gguf.InvalidModelError, "magic"),
    ({"version": 2}, UnsupportedError, "gguf_version"),
    ({"bad_offset": True}, gguf.InvalidModelError, "not aligned"),
])
def test_header_errors(tmp_path, kw, exc, needle):
    p = tmp_path / "bad.gguf"
    write_gguf(p, [("w", [256, 2], 12, blocks(12, 2, 256).tobytes())], **kw)
    with pytest.raises(exc) as e:
        gguf.inspect(p)
    assert needle in str(e.value)


def test_truncated_payload_is_rejected(tmp_path):
    p = tmp_path / "t.gguf"
    write_gguf(p, [("w", [256, 4], 12, blocks(12, 4, 256).tobytes())])
    data = p.read_bytes()
    p.write_bytes(data[:-200])
    with pytest.raises(gguf.InvalidModelError) as e:
        gguf.inspect(p)
    assert "exceeds file length" in str(e.value)


def test_interop_with_gguf_package_writer(tmp_path):
    ggufpkg = pytest.importorskip("gguf")
    q4 = blocks(12, 16, 512)
    p = tmp_path / "pkg.gguf"
    w = ggufpkg.GGUFWriter(str(p), "llama")
    w.add_tensor("w", q4.reshape(16, 2 * 144),
                 raw_dtype=ggufpkg.GGMLQuantizationType.Q4_K)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    m = gguf.inspect(p)
    t = m.tensor("w")
    assert (t.k, t.n_rows, t.tensor_type) == (512, 16, 12)
    assert np.array_equal(gguf.read_payload(m, "w"), q4)
