"""GPU: the quantized linear layers of a GGUF decoder (fused qkv + bias, o, fused
gated MLP, Q8_0 embedding, head + greedy argmax) vs the CPU oracle
(the quantized counterpart of crates/models/src/qwen/qwen2_5/weights.rs:150-224)."""
import numpy as np
import pytest
import torch

from tests.tolerance import GEMV_RTOL, normwise_err, rel_err

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model_file(tmp_path_factory):
    from tests.gguf_writer import write_gguf
    from tests.model_files import decoder_tensors
    t = decoder_tensors()
    f = tmp_path_factory.mktemp("m") / "decoder.gguf"
    write_gguf(f, t)
    return f, t


@pytest.mark.parametrize("rows", [1, 3])
def test_decoder_linears_match_oracle(backend, oracle, model_file, rows):
    from ocelotl_b200 import gguf, synth
    from ocelotl_b200.model import QuantizedDecoderLinears
    from tests.model_files import H, I, KV, Q, V, payload
    f, tensors = model_file
    model = QuantizedDecoderLinears(backend, gguf.inspect(f))
    x = synth.activations(rows, H, 7, "mx").numpy()
    xd = torch.from_numpy(x).cuda()
    for i in range(2):
        p = f"blk.{i}."
        # fused q/k/v (+ bias) == the three projections run separately
        y = torch.empty(rows, Q + 2 * KV, device="cuda")
        model.qkv(i, xd, rows, y)
        backend.synchronize()
        parts = []
        for s, n in zip("qkv", (Q, KV, KV)):
            t, blocks = payload(tensors, p + f"attn_{s}.weight")
            _, b = payload(tensors, p + f"attn_{s}.bias")
            parts.append(oracle.q_linear(t, blocks, x, rows, H, n, bias=b.view(np.float32)))
        assert rel_err(y.cpu().numpy(), np.concatenate(parts, axis=1)) <= GEMV_RTOL
        # o
        yo = torch.empty(rows, H, device="cuda")
        model.o(i, xd, rows, yo)
        backend.synchronize()
        t, blocks = payload(tensors, p + "attn_output.weight")
        assert rel_err(yo.cpu().numpy(), oracle.q_linear(t, blocks, x, rows, Q, H)) <= GEMV_RTOL
        # gated MLP
        act = torch.empty(rows * I, device="cuda")
        out = torch.empty(rows * H, device="cuda")
        model.mlp(i, xd, rows, act, out)
        backend.synchronize()
        tg, gb = payload(tensors, p + "ffn_gate.weight")
        _, ub = payload(tensors, p + "ffn_up.weight")
        td, db = payload(tensors, p + "ffn_down.weight")
        ref_act, ref_out = oracle.q_mlp_gated_silu(tg, gb, ub, td, db, x, rows, H, I)
        a = act.cpu().numpy().reshape(rows, I)
        assert rel_err(a, ref_act) <= 2 * GEMV_RTOL
        assert normwise_err(out.cpu().numpy().reshape(rows, H), ref_out) <= 2e-3
    # embedding rows and the head + greedy argmax
    ids = torch.tensor([0, 17, V - 1][:rows], dtype=torch.int32, device="cuda")
    h = model.embed(ids)
    backend.synchronize()
    te, eb = payload(tensors, "token_embd.weight")
    table = oracle.dequant(te, eb, V, H)
    assert np.array_equal(h.cpu().numpy().view(np.uint32), table[ids.cpu().numpy()].view(np.uint32))
    next_ids, logits = model.head_argmax(h, rows)
    backend.synchronize()
    th, hb = payload(tensors, "output.weight")
    ref_logits = oracle.q_linear(th, hb, h.cpu().numpy(), rows, H, V)
    assert rel_err(logits.cpu().numpy(), ref_logits) <= GEMV_RTOL
    got = next_ids.cpu().numpy()
    for r in range(rows):
        assert got[r] == oracle.greedy_sample_fast(logits.cpu().numpy()[r])
    assert backend.take_device_errors() == (0, 0)
