"""Small synthetic GGUF decoder files for the model-linear tests."""
import numpy as np

H, Q, KV, I, V = 256, 256, 64, 512, 1000


def decoder_tensors(n_layers=2, bias=True, tied=False, qkv_types=(12, 12, 12), seed=3):
    from ocelotl_b200 import synth
    t = []

    def q(name, typ, rows, k):
        blocks = synth.quant_blocks(typ, rows, k, seed, name).numpy()
        t.append((name, [k, rows], typ, blocks.tobytes()))
        return blocks

    q("token_embd.weight", 8, V, H)
    if not tied:
        q("output.weight", 14, V, H)
    for i in range(n_layers):
        p = f"blk.{i}."
        for s, rows, typ in zip("qkv", (Q, KV, KV), qkv_types):
            q(p + f"attn_{s}.weight", typ, rows, H)
            if bias:
                b = synth.activations(1, rows, seed, p + s + "b").numpy().reshape(-1).astype(np.float32)
                t.append((p + f"attn_{s}.bias", [rows], 0, b.tobytes()))
        q(p + "attn_output.weight", 12, H, Q)
        q(p + "ffn_gate.weight", 12, I, H)
        q(p + "ffn_up.weight", 12, I, H)
        q(p + "ffn_down.weight", 14, H, I)
    return t


def payload(tensors, name):
    for n, shape, typ, data in tensors:
        if n == name:
            return typ, np.frombuffer(data, dtype=np.uint8)
    raise KeyError(name)
