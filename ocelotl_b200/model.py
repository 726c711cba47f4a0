"""Quantized linear layers of a Llama / Qwen-style decoder, loaded from a GGUF file.

The reference's Qwen2.5 loader keeps every projection as a pre-transposed f32
matrix and runs it through `matmul` (crates/models/src/qwen/qwen2_5/weights.rs:
150-224: q/k/v with biases, o, gate/up/down per layer; embed_tokens; the head).
This module is the quantized path for the same layers: the GGUF tensors stay
quantized in HBM and run through the fused dequant-GEMV (`linear_d`), with

* q, k and v fused into one weight (their GGUF rows concatenated: rows are
  independent block runs, so concatenation is a byte concatenation) and their
  f32 biases concatenated -- one activation split and one launch per layer;
* gate and up interleaved into one pair for the fused gated MLP
  (`mlp_gated_silu`: silu(gate) * up, then down);
* the output head as a GEMV over the vocabulary followed by greedy argmax on
  the device (`greedy_sample`), the embedding as a Q8_0 row gather.

Tensor names follow the GGUF convention for these models (token_embd.weight,
blk.N.attn_{q,k,v}.{weight,bias}, blk.N.attn_output.weight,
blk.N.ffn_{gate,up,down}.weight, output.weight; a missing head is tied to the
embedding table).  Attention, norms and rotary embeddings are not part of this
path; the caller runs them between the projections.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from .errors import InvalidRequestError, UnsupportedError
from .ggml import GgmlType
from .gguf import Manifest, TensorEntry, read_payload

QUANT_TYPES = (GgmlType.Q4_K, GgmlType.Q6_K, GgmlType.Q8_0)
F32 = 0


@dataclass
class LayerPlan:
    """Which GGUF tensors make up one decoder layer's linear projections."""
    index: int
    qkv: list[str]               # q, k, v weights fused in this order
    qkv_bias: list[str]          # their f32 biases (empty if none)
    qkv_rows: list[int]          # output rows of q, k, v
    o: str
    gate: str
    up: str
    down: str


@dataclass
class ModelPlan:
    hidden: int
    intermediate: int
    vocab: int
    embed: str
    head: str                    # == embed when the head is tied
    layers: list[LayerPlan] = field(default_factory=list)


def _need(m: Manifest, name: str) -> TensorEntry:
    try:
        return m.tensor(name)
    except InvalidRequestError:
        raise InvalidRequestError("tensor", f"GGUF file {m.path} has no tensor `{name}`") from None


def _quant(t: TensorEntry) -> None:
    if t.tensor_type not in QUANT_TYPES:
        raise UnsupportedError("quantized weight type", f"{t.name}: {t.tensor_type}",
                               ["Q4_K(12)", "Q6_K(14)", "Q8_0(8)"])


def plan(m: Manifest, n_layers: int | None = None) -> ModelPlan:
    """Map a GGUF manifest to the decoder's linear layers (host only, reads no payload)."""
    emb = _need(m, "token_embd.weight")
    hidden, vocab = emb.k, emb.n_rows
    names = {t.name for t in m.tensors}
    head = "output.weight" if "output.weight" in names else "token_embd.weight"
    count = 0
    while f"blk.{count}.attn_q.weight" in names:
        count += 1
    if n_layers is not None:
        if n_layers > count:
            raise InvalidRequestError("n_layers", f"requested {n_layers} layers, the file has {count}")
        count = n_layers
    out = None
    for i in range(count):
        p = f"blk.{i}."
        ws = [_need(m, p + f"attn_{s}.weight") for s in ("q", "k", "v")]
        for w in ws:
            _quant(w)
            if w.k != hidden:
                raise InvalidRequestError("tensor", f"`{w.name}` in_features {w.k} != hidden {hidden}")
        bias = [p + f"attn_{s}.bias" for s in ("q", "k", "v") if p + f"attn_{s}.bias" in names]
        if bias and len(bias) != 3:
            raise InvalidRequestError("tensor", f"layer {i}: q/k/v biases must be all present or all absent")
        for b in bias:
            if _need(m, b).tensor_type != F32:
                raise UnsupportedError("bias type", f"{b}: {_need(m, b).tensor_type}", ["F32(0)"])
        if len({w.tensor_type for w in ws}) != 1:  # fusion concatenates rows of one block format
            raise UnsupportedError("q/k/v of different quant types", str([int(w.tensor_type) for w in ws]),
                                   ["one type for q, k and v"])
        gate, up, down = (_need(m, p + f"ffn_{s}.weight") for s in ("gate", "up", "down"))
        for w in (gate, up, down):
            _quant(w)
        if gate.tensor_type != up.tensor_type or gate.n_rows != up.n_rows or gate.k != up.k:
            raise InvalidRequestError("tensor", f"layer {i}: ffn_gate and ffn_up differ in type or shape")
        if down.k != gate.n_rows or down.n_rows != hidden:
            raise InvalidRequestError("tensor", f"layer {i}: ffn_down is [{down.n_rows} x {down.k}], expected "
                                                f"[{hidden} x {gate.n_rows}]")
        o = _need(m, p + "attn_output.weight")
        _quant(o)
        lp = LayerPlan(i, [w.name for w in ws], bias, [w.n_rows for w in ws], o.name, gate.name, up.name,
                       down.name)
        if out is None:
            out = ModelPlan(hidden, gate.n_rows, vocab, emb.name, head)
        elif gate.n_rows != out.intermediate:
            raise InvalidRequestError("tensor", f"layer {i}: intermediate {gate.n_rows} != {out.intermediate}")
        out.layers.append(lp)
    if out is None:
        out = ModelPlan(hidden, 0, vocab, emb.name, head)
    _quant(_need(m, head))
    return out


def fused_qkv_payload(m: Manifest, lp: LayerPlan) -> tuple[int, np.ndarray, int]:
    """(type, concatenated GGUF rows of q, k, v, total rows)."""
    ts = [m.tensor(n) for n in lp.qkv]
    blob = np.concatenate([np.ascontiguousarray(read_payload(m, t.name)) for t in ts])
    return ts[0].tensor_type, blob, sum(t.n_rows for t in ts)


class QuantizedDecoderLinears:
    """Every linear layer of the decoder resident in HBM, quantized.

    Per layer: `qkv(x, rows, out)` -> [rows, q+k+v] (bias added), `o(...)`,
    `mlp(x, rows, act, out)` (silu(gate)*up then down); plus `embed(ids, out)`
    and `head_argmax(h, rows)` -> next token ids on the device.  x / out are
    contiguous f32 torch tensors on the backend's device.
    """

    def __init__(self, backend, manifest: Manifest, n_layers: int | None = None):
        import torch

        from .gguf import upload_quant_tensor
        self.backend = backend
        self.plan = plan(manifest, n_layers)
        dev = backend.torch_device
        self.layers = []
        for lp in self.plan.layers:
            t, blob, rows = fused_qkv_payload(manifest, lp)
            qkv = backend.upload_quant(t, blob, rows, self.plan.hidden)
            bias = None
            if lp.qkv_bias:
                bias = torch.from_numpy(np.concatenate(
                    [np.frombuffer(bytes(read_payload(manifest, b)), dtype=np.float32) for b in lp.qkv_bias])).to(dev)
            gate = upload_quant_tensor(backend, manifest, lp.gate)
            up = upload_quant_tensor(backend, manifest, lp.up)
            pair = backend.pair_gated(gate, up)
            gate.quant.free()
            up.quant.free()
            self.layers.append({
                "qkv": qkv, "qkv_bias": bias, "qkv_rows": lp.qkv_rows,
                "o": upload_quant_tensor(backend, manifest, lp.o),
                "gate_up": pair,
                "down": upload_quant_tensor(backend, manifest, lp.down),
            })
        self.embed_table = upload_quant_tensor(backend, manifest, self.plan.embed)
        self.head_w = self.embed_table if self.plan.head == self.plan.embed else \
            upload_quant_tensor(backend, manifest, self.plan.head)

    # -- per layer ----------------------------------------------------------
    def qkv(self, i: int, x, rows: int, out) -> None:
        L = self.layers[i]
        self.backend.linear_dev(L["qkv"], x, rows, out, bias=L["qkv_bias"])

    def o(self, i: int, x, rows: int, out) -> None:
        self.backend.linear_dev(self.layers[i]["o"], x, rows, out)

    def mlp(self, i: int, x, rows: int, act, out) -> None:
        L = self.layers[i]
        self.backend.mlp_gated_silu(x, rows, self.plan.hidden, self.plan.intermediate, L["gate_up"], None,
                                    L["down"], act, None, out)

    # -- model ends ---------------------------------------------------------
    def embed(self, ids, out=None):
        return self.backend.embed_rows(self.embed_table, ids, out)

    def head_argmax(self, h, rows: int, logits=None, ids=None):
        import torch
        if logits is None:
            logits = torch.empty(rows, self.plan.vocab, device=self.backend.torch_device)
        self.backend.linear_dev(self.head_w, h, rows, logits)
        return self.backend.greedy_sample(logits, out=ids), logits
