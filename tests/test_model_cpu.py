"""CPU: mapping a GGUF decoder's tensors to the quantized linear layers (no GPU)."""
import pytest

from ocelotl_b200 import gguf
from ocelotl_b200.errors import InvalidRequestError, UnsupportedError
from ocelotl_b200.model import plan
from tests.gguf_writer import write_gguf
from tests.model_files import H, I, KV, Q, V, decoder_tensors


def test_plan_maps_layers_and_fuses_qkv(tmp_path):
    f = tmp_path / "m.gguf"
    write_gguf(f, decoder_tensors())
    p = plan(gguf.inspect(f))
    assert (p.hidden, p.intermediate, p.vocab) == (H, I, V)
    assert p.head == "output.weight" and p.embed == "token_embd.weight"
    assert len(p.layers) == 2
    lp = p.layers[1]
    assert lp.qkv == ["blk.1.attn_q.weight", "blk.1.attn_k.weight", "blk.1.attn_v.weight"]
    assert lp.qkv_rows == [Q, KV, KV] and len(lp.qkv_bias) == 3
    assert (lp.o, lp.gate, lp.up, lp.down) == ("blk.1.attn_output.weight", "blk.1.ffn_gate.weight",
                                               "blk.1.ffn_up.weight", "blk.1.ffn_down.weight")
    assert len(plan(gguf.inspect(f), n_layers=1).layers) == 1
    with pytest.raises(InvalidRequestError):
        plan(gguf.inspect(f), n_layers=3)


def test_tied_head_and_no_bias(tmp_path):
    f = tmp_path / "t.gguf"
    write_gguf(f, decoder_tensors(n_layers=1, bias=False, tied=True))
    p = plan(gguf.inspect(f))
    assert p.head == p.embed == "token_embd.weight"
    assert p.layers[0].qkv_bias == []


def test_mixed_qkv_types_are_unsupported(tmp_path):
    f = tmp_path / "x.gguf"
    write_gguf(f, decoder_tensors(n_layers=1, qkv_types=(12, 14, 12)))
    with pytest.raises(UnsupportedError):
        plan(gguf.inspect(f))


def test_missing_tensor_is_named(tmp_path):
    f = tmp_path / "y.gguf"
    write_gguf(f, [t for t in decoder_tensors(n_layers=1) if t[0] != "blk.0.ffn_up.weight"])
    with pytest.raises(InvalidRequestError, match="ffn_up"):
        plan(gguf.inspect(f))
