"""Seeded synthesis of ggmlc-format GGUF decoder models (fixture builder for bench and tests).

Writes the same container the reference compiler produces for a Llama-family model wrapped by
``examples/models/hub_models.py:load_smollm2_model`` and compiled with ``ggmlc.compile(...,
quantize="q8_0"|"q4_0", dynamic_shapes=Dim("s"))``: GGUF v3 (python/ggmlc/serialization/
gguf.py:288-366, 32-byte alignment) with a ``ggmlc.graph_spec`` JSON whose node sequence per
layer is RMS_NORM(202) -> MUL_MAT(fused QKV) -> VIEW x3 -> RESHAPE x3 -> PERMUTE(v) -> ROPE x2
-> PERMUTE x2 -> FLASH_ATTN_EXT -> RESHAPE -> MUL_MAT(o) -> ADD -> RMS_NORM -> MUL_MAT(fused
gate_up) -> SWIGLU(203) -> MUL_MAT(down) -> ADD, closed by RMS_NORM(+gamma) -> MUL_MAT(tied
embedding).  tests/test_synth.py checks the structure against a reference-compiled fixture.

Weights are N(0, 0.02) from a seed, quantized with the compile-time quantizers of
python/ggmlc/quantization/quantize.py (Q8_0 :10-47, Q4_0 :65-107), restated below; on a CUDA
box torch does the generation and quantization (same float64 arithmetic) so the 8B/70B shapes
take seconds.  RMS gammas are 1 (a random-init HF model), which the RMS-gamma bake folds away.
"""

from __future__ import annotations

import json
import struct
from dataclasses import dataclass
from pathlib import Path
from typing import Callable, Iterator

import numpy as np

Q8_0, Q4_0, F32, I32 = 8, 2, 0, 26
BLOCK = 32
ALIGN = 32


@dataclass
class LlamaShape:
    n_layers: int
    d_model: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    rope_theta: float = 10000.0
    eps: float = 1e-5
    max_seq: int = 2048


@dataclass
class GPT2Shape:
    n_layers: int
    d_model: int
    n_heads: int
    ffn: int
    vocab: int
    n_pos: int
    eps: float = 1e-5


SHAPES = {
    # the shapes of the benchmark configurations: SmolLM2-135M, Llama-3-8B / 70B, GPT-2-small
    "smollm2-135m": LlamaShape(30, 576, 9, 3, 64, 1536, 49152, 10000.0),
    "llama3-8b": LlamaShape(32, 4096, 32, 8, 128, 14336, 128256, 500000.0),
    "llama3-70b": LlamaShape(80, 8192, 64, 8, 128, 28672, 128256, 500000.0),
    "gpt2-small": GPT2Shape(12, 768, 12, 3072, 50257, 1024),
}


# ------------------------------------------------------------------------------ quantizers

def quantize_q8_0_np(x: np.ndarray) -> np.ndarray:
    """_quantize_q8_0_chunk (quantize.py:10-25): scale = max|x|/127 (float64) -> fp16,
    q = clip(round(x * float32(1/scale)), -128, 127)."""
    b = np.ascontiguousarray(x, np.float32).reshape(-1, BLOCK)
    mx = np.max(np.abs(b), axis=1)
    scale = np.where(mx > 0, mx / 127.0, 0.0)
    s16 = scale.astype(np.float16)
    safe = np.where(scale != 0, scale, 1.0)[:, None]
    inv = (1.0 / safe).astype(np.float32)
    q = np.clip(np.round(b * inv), -128, 127).astype(np.int8)
    return np.hstack([s16.view(np.uint8).reshape(-1, 2), q.view(np.uint8)]).reshape(-1)


def quantize_q4_0_np(x: np.ndarray) -> np.ndarray:
    """quantize_q4_0 (quantize.py:65-107): scale = signed_max / -8 (float64) -> fp16,
    q = clip(round(x / scale) + 8, 0, 15), low nibble = element j, high = element j+16."""
    b = np.ascontiguousarray(x, np.float32).reshape(-1, BLOCK)
    n = b.shape[0]
    idx = np.argmax(np.abs(b), axis=1)
    smax = b[np.arange(n), idx]
    scale = np.where(smax != 0, smax / -8.0, 0.0)
    s16 = scale.astype(np.float16)
    safe = np.where(scale != 0, scale, 1.0)[:, None]
    q = np.where(scale[:, None] != 0, np.clip(np.round(b / safe) + 8, 0, 15), 8).astype(np.uint8)
    packed = (q[:, :16] & 0x0F) | ((q[:, 16:] & 0x0F) << 4)
    return np.hstack([s16.view(np.uint8).reshape(-1, 2), packed.astype(np.uint8)]).reshape(-1)


def _quantize_torch(x, qtype: int) -> np.ndarray:
    """Same arithmetic as the numpy quantizers, on a torch device."""
    import torch

    b = x.reshape(-1, BLOCK).to(torch.float32)
    if qtype == Q8_0:
        mx = b.abs().amax(dim=1).to(torch.float64)
        scale = torch.where(mx > 0, mx / 127.0, torch.zeros_like(mx))
        s16 = scale.to(torch.float16)
        safe = torch.where(scale != 0, scale, torch.ones_like(scale))
        inv = (1.0 / safe).to(torch.float32)[:, None]
        q = torch.clamp(torch.round(b * inv), -128, 127).to(torch.int8)
        out = torch.cat([s16.view(torch.uint8).reshape(-1, 2), q.view(torch.uint8)], dim=1)
    else:
        idx = b.abs().argmax(dim=1)
        smax = b.gather(1, idx[:, None])[:, 0].to(torch.float64)
        scale = torch.where(smax != 0, smax / -8.0, torch.zeros_like(smax))
        s16 = scale.to(torch.float16)
        safe = torch.where(scale != 0, scale, torch.ones_like(scale))[:, None]
        q = torch.where(scale[:, None] != 0,
                        torch.clamp(torch.round(b.to(torch.float64) / safe) + 8, 0, 15),
                        torch.full_like(b, 8, dtype=torch.float64)).to(torch.uint8)
        packed = (q[:, :16] & 0x0F) | ((q[:, 16:] & 0x0F) << 4)
        out = torch.cat([s16.view(torch.uint8).reshape(-1, 2), packed], dim=1)
    return out.reshape(-1).cpu().numpy()


def quantized_normal(shape_rows: int, cols: int, qtype: int, seed: int, std: float = 0.02,
                     device: str | None = None) -> Iterator[np.ndarray]:
    """Yields the GGUF block bytes of an N(0, std) [rows, cols] matrix in row chunks."""
    chunk = max(1, (64 << 20) // max(cols, 1))
    if device:
        import torch

        g = torch.Generator(device=device)
        g.manual_seed(seed)
        for r0 in range(0, shape_rows, chunk):
            n = min(chunk, shape_rows - r0)
            x = torch.randn((n, cols), generator=g, device=device, dtype=torch.float32) * std
            yield _quantize_torch(x, qtype)
    else:
        rng = np.random.default_rng(seed)
        for r0 in range(0, shape_rows, chunk):
            n = min(chunk, shape_rows - r0)
            x = (rng.standard_normal((n, cols), dtype=np.float32) * std).astype(np.float32)
            yield quantize_q8_0_np(x) if qtype == Q8_0 else quantize_q4_0_np(x)


# ------------------------------------------------------------------------------ graph spec

def _dim(v) -> dict:
    return {"type": "symbol", "name": v} if isinstance(v, str) else {"type": "static", "val": int(v)}


def rope_freq_base(theta: float, head_dim: int) -> float:
    """freq_base as the fusion pass recovers it from the wrapper's inv_freq buffer
    (fusion.py:322: (1/inv_freq[1]) ** (n_dims/2) in float32).  The buffer is built with torch's
    float32 pow, as the wrapper builds it (examples/models/hub_models.py:303): numpy's float32
    power differs from it by an ulp at theta 500000, which the recovery's power of n_dims/2
    turns into a freq_base about 1.25 apart."""
    import torch

    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    inv = inv.numpy().astype(np.float32)
    return float(np.power(np.float32(1.0) / inv[1], np.float32(head_dim / 2.0)))


def llama_graph(cfg: LlamaShape, qtype: int, name: str, sym: str = "s70"):
    """Returns (spec dict, tensor list [(name, ne, type, maker)]) for a Llama-family model."""
    tensors: dict[str, dict] = {}
    nodes: list[dict] = []
    params: list[int] = []
    payload: list[tuple] = []
    nid = [0]
    tid = [0]

    def tensor(tname, ne, ttype, storage, role=None, producer=None, data=None):
        i = tid[0]
        tid[0] += 1
        tensors[str(i)] = {"id": i, "name": tname, "type": ttype,
                           "ne": [_dim(v) for v in (list(ne) + [1] * (4 - len(ne)))],
                           "storage": storage, "producer_id": producer, "role": role}
        if data is not None:
            payload.append((tname, [v for v in ne], ttype, data))
            if storage == 1:
                params.append(i)
        return i

    def node(opcode, inputs, out_name, out_ne, attrs, op_name, storage=3):
        i = nid[0]
        nid[0] += 1
        out = tensor(out_name, out_ne, F32, storage, producer=i)
        nodes.append({"id": i, "opcode": opcode, "inputs": inputs, "outputs": [out],
                      "attributes": attrs, "name": op_name})
        return out

    d, hq, hkv, hd, ffn, V, L = (cfg.d_model, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn,
                                 cfg.vocab, cfg.n_layers)
    s = sym
    qkv_n = (hq + 2 * hkv) * hd
    seed = [1000]

    def wmaker(rows, cols):
        seed[0] += 1
        sd = seed[0]
        return lambda device: quantized_normal(rows, cols, qtype, sd, device=device)

    emb = tensor("embed_tokens.weight", [d, V], qtype, 1, data=wmaker(V, d))
    ids = tensor("input_ids", [s], I32, 0, role="input")
    ar = tensor("arange", [s], I32, 2, role="constant",
                data=lambda device: iter([np.arange(cfg.max_seq, dtype=np.int32).view(np.uint8)]))
    fb = rope_freq_base(cfg.rope_theta, hd)
    eps = float(np.float32(cfg.eps))
    x = node(40, [emb, ids], "embedding", [d, s], {"source_op": "aten.embedding.default"}, "embedding")
    for li in range(L):
        p = f"layers.{li}."
        wqkv = tensor(p + "self_attn.fused_qkv.weight", [d, qkv_n], qtype, 1, data=wmaker(qkv_n, d))
        wo = tensor(p + "self_attn.o_proj.weight", [hq * hd, d], qtype, 1, data=wmaker(d, hq * hd))
        wgu = tensor(p + "mlp.fused_gate_up.weight", [d, 2 * ffn], qtype, 1, data=wmaker(2 * ffn, d))
        wdn = tensor(p + "mlp.down_proj.weight", [ffn, d], qtype, 1, data=wmaker(d, ffn))
        h = node(202, [x], f"l{li}_norm1", [d, s], {"eps": eps, "fused_pass": "RMSNorm Normalization Fusion"}, f"l{li}_rms1")
        qkv = node(29, [wqkv, h], f"l{li}_qkv", [qkv_n, s], {"fused_pass": "Horizontal QKV Projection Fusion"}, f"l{li}_qkv")
        sl = []
        for j, (a, b) in enumerate([(0, hq * hd), (hq * hd, (hq + hkv) * hd), ((hq + hkv) * hd, qkv_n)]):
            sl.append(node(37, [qkv], f"l{li}_slice{j}", [b - a, s],
                           {"dim": -1, "start": a, "end": b, "step": 1, "ggml_dim": 0}, f"l{li}_slice{j}"))
        qv = node(36, [sl[0]], f"l{li}_q", [hd, hq, s, 1], {"shape": [1, s, hq, hd]}, f"l{li}_view_q")
        kv_ = node(36, [sl[1]], f"l{li}_k", [hd, hkv, s, 1], {"shape": [1, s, hkv, hd]}, f"l{li}_view_k")
        vv = node(36, [sl[2]], f"l{li}_v", [hd, hkv, s, 1], {"shape": [1, s, hkv, hd]}, f"l{li}_view_v")
        perm = {"dim0": 1, "dim1": 2, "axis0": 0, "axis1": 2, "axis2": 1, "axis3": 3}
        vt = node(38, [vv], f"l{li}_vt", [hd, s, hkv, 1], dict(perm), f"l{li}_vt")
        rope = {"n_dims": hd, "mode": 2, "freq_base": fb, "freq_scale": 1.0}
        qr = node(48, [qv, ar], f"l{li}_qrope", [hd, hq, s, 1], dict(rope), f"l{li}_qrope")
        qt = node(38, [qr], f"l{li}_qt", [hd, s, hq, 1], dict(perm), f"l{li}_qt")
        kr = node(48, [kv_, ar], f"l{li}_krope", [hd, hkv, s, 1], dict(rope), f"l{li}_krope")
        kt = node(38, [kr], f"l{li}_kt", [hd, s, hkv, 1], dict(perm), f"l{li}_kt")
        att = node(74, [qt, kt, vt], f"l{li}_attn", [hd, hq, s, 1],
                   {"is_causal": 1, "enable_gqa": True, "fused_transpose": 1}, f"l{li}_sdpa")
        a2 = node(36, [att], f"l{li}_attn2d", [hq * hd, s], {"shape": [1, s, "-1"]}, f"l{li}_view_o")
        o = node(29, [wo, a2], f"l{li}_o", [d, s], {}, f"l{li}_o_proj")
        x = node(2, [x, o], f"l{li}_res1", [d, s], {}, f"l{li}_add1")
        h2 = node(202, [x], f"l{li}_norm2", [d, s], {"eps": eps, "fused_pass": "RMSNorm Normalization Fusion"}, f"l{li}_rms2")
        gu = node(29, [wgu, h2], f"l{li}_gate_up", [2 * ffn, s], {"fused_pass": "Horizontal GATE_UP Projection Fusion"}, f"l{li}_gate_up")
        act = node(203, [gu], f"l{li}_swiglu", [ffn, s], {"fused_pass": "SwiGLU Activation Fusion (silu(gate) * up)"}, f"l{li}_swiglu")
        dn = node(29, [wdn, act], f"l{li}_down", [d, s], {}, f"l{li}_down_proj")
        x = node(2, [x, dn], f"l{li}_res2", [d, s], {}, f"l{li}_add2")
    gam = tensor("norm.weight", [d], F32, 1, role="parameter",
                 data=lambda device: iter([np.ones(d, np.float32).view(np.uint8)]))
    hf = node(202, [x, gam], "final_norm", [d, s], {"eps": eps, "fused_pass": "RMSNorm Normalization Fusion"}, "final_rms")
    logits = node(29, [emb, hf], "logits", [V, s], {}, "lm_head", storage=5)
    spec = {"name": name, "inputs": [ids], "outputs": [logits], "parameters": sorted(params),
            "symbol_table": [s], "metadata": {}, "tensors": tensors, "nodes": nodes}
    return spec, payload


def gpt2_graph(cfg: GPT2Shape, qtype: int, name: str, sym: str = "s70"):
    """(spec, payload) of a GPT-2 model as the reference compiler emits it for the
    ``examples/models/hub_models.py:load_gpt2_model`` wrapper: token + learned position
    embeddings, per layer LAYER_NORM(201, affine baked into the next linear) -> MUL_MAT(fused
    QKV + bias) -> SLICE x3 -> (VIEW, PERMUTE) x3 -> FLASH_ATTN_EXT -> VIEW -> MUL_MAT(out_proj +
    bias) -> ADD -> LAYER_NORM -> MUL_MAT(mlp_fc + baked bias) -> BIAS_GELU(200, tanh) ->
    MUL_MAT(mlp_proj + bias) -> ADD, closed by LAYER_NORM(ln_f gamma, beta) -> MUL_MAT(tied wte).
    Random init as the config asks: matrices N(0, 0.02), biases 0, LayerNorm gamma 1 beta 0 (the
    bake then leaves the fused biases 0)."""
    tensors: dict[str, dict] = {}
    nodes: list[dict] = []
    params: list[int] = []
    payload: list[tuple] = []
    nid = [0]
    tid = [0]

    def tensor(tname, ne, ttype, storage, role=None, producer=None, data=None):
        i = tid[0]
        tid[0] += 1
        tensors[str(i)] = {"id": i, "name": tname, "type": ttype,
                           "ne": [_dim(v) for v in (list(ne) + [1] * (4 - len(ne)))],
                           "storage": storage, "producer_id": producer, "role": role}
        if data is not None:
            payload.append((tname, [v for v in ne], ttype, data))
            if storage == 1:
                params.append(i)
        return i

    def node(opcode, inputs, out_name, out_ne, attrs, op_name, storage=3):
        i = nid[0]
        nid[0] += 1
        out = tensor(out_name, out_ne, F32, storage, producer=i)
        nodes.append({"id": i, "opcode": opcode, "inputs": inputs, "outputs": [out],
                      "attributes": attrs, "name": op_name})
        return out

    d, H, F, V, L = cfg.d_model, cfg.n_heads, cfg.ffn, cfg.vocab, cfg.n_layers
    hd = d // H
    s = sym
    seed = [2000]

    def wmaker(rows, cols):
        seed[0] += 1
        sd = seed[0]
        return lambda device: quantized_normal(rows, cols, qtype, sd, device=device)

    def zeros(n):
        return lambda device: iter([np.zeros(n, np.float32).view(np.uint8)])

    wte = tensor("wte.weight", [d, V], qtype, 1, data=wmaker(V, d))
    wpe = tensor("wpe.weight", [d, cfg.n_pos], qtype, 1, data=wmaker(cfg.n_pos, d))
    ids = tensor("input_ids", [s], I32, 0, role="input")
    pids = tensor("position_ids", [s], I32, 0, role="input")
    eps = float(cfg.eps)
    e0 = node(40, [wte, ids], "embedding", [d, s], {"source_op": "aten.embedding.default"}, "embedding")
    e1 = node(40, [wpe, pids], "embedding_1", [d, s], {"source_op": "aten.embedding.default"}, "embedding_1")
    x = node(2, [e0, e1], "add", [d, s], {"source_op": "aten.add.Tensor"}, "add")
    perm = {"dim0": 1, "dim1": 2, "axis0": 0, "axis1": 2, "axis2": 1, "axis3": 3}
    for li in range(L):
        p = f"layers.{li}."
        wqkv = tensor(p + "fused_qkv.weight", [d, 3 * d], qtype, 1, data=wmaker(3 * d, d))
        bqkv = tensor(p + "fused_qkv.bias", [3 * d], F32, 1, data=zeros(3 * d))
        wo = tensor(p + "out_proj.weight", [d, d], qtype, 1, data=wmaker(d, d))
        bo = tensor(p + "out_proj.bias", [d], F32, 1, role="parameter", data=zeros(d))
        wfc = tensor(p + "mlp_fc.weight", [d, F], qtype, 1, data=wmaker(F, d))
        # the bake names the folded bias after the linear node it feeds (linear_4, linear_10, ...)
        bfc_baked = tensor(f"linear_{6 * li + 4}_baked_bias", [F], F32, 1, role="bias",
                           data=zeros(F))
        bfc = tensor(p + "mlp_fc.bias", [F], F32, 1, role="parameter", data=zeros(F))
        wpj = tensor(p + "mlp_proj.weight", [F, d], qtype, 1, data=wmaker(d, F))
        bpj = tensor(p + "mlp_proj.bias", [d], F32, 1, role="parameter", data=zeros(d))
        h = node(201, [x], f"l{li}_ln1", [d, s], {"eps": eps}, f"l{li}_ln1")
        qkv = node(29, [wqkv, h, bqkv], f"l{li}_qkv", [3 * d, s],
                   {"fused_pass": "Horizontal QKV Projection Fusion"}, f"l{li}_qkv")
        sl = [node(37, [qkv], f"l{li}_slice{j}", [d, s],
                   {"dim": -1, "start": j * d, "end": (j + 1) * d, "step": 1, "ggml_dim": 0},
                   f"l{li}_slice{j}") for j in range(3)]
        hv = []
        for j in range(3):
            v_ = node(36, [sl[j]], f"l{li}_view{j}", [hd, H, s, 1], {"shape": [1, s, H, hd]},
                      f"l{li}_view{j}")
            hv.append(node(38, [v_], f"l{li}_t{j}", [hd, s, H, 1], dict(perm), f"l{li}_t{j}"))
        att = node(74, hv, f"l{li}_attn", [hd, H, s, 1], {"is_causal": 1, "fused_transpose": 1},
                   f"l{li}_sdpa")
        a2 = node(36, [att], f"l{li}_attn2d", [d, s], {"shape": [1, s, "-1"]}, f"l{li}_view_o")
        o = node(29, [wo, a2, bo], f"l{li}_o", [d, s], {}, f"l{li}_out_proj")
        x = node(2, [x, o], f"l{li}_res1", [d, s], {}, f"l{li}_add1")
        h2 = node(201, [x], f"l{li}_ln2", [d, s], {"eps": eps}, f"l{li}_ln2")
        fc = node(29, [wfc, h2, bfc_baked], f"l{li}_fc", [F, s], {}, f"l{li}_mlp_fc")
        g = node(200, [fc, bfc], f"l{li}_gelu", [F, s], {"approximate": "tanh"}, f"l{li}_gelu")
        pj = node(29, [wpj, g, bpj], f"l{li}_proj", [d, s], {}, f"l{li}_mlp_proj")
        x = node(2, [x, pj], f"l{li}_res2", [d, s], {}, f"l{li}_add2")
    gam = tensor("ln_f.weight", [d], F32, 1, role="parameter",
                 data=lambda device: iter([np.ones(d, np.float32).view(np.uint8)]))
    bet = tensor("ln_f.bias", [d], F32, 1, role="parameter", data=zeros(d))
    hf = node(201, [x, gam, bet], "final_ln", [d, s], {"eps": eps}, "final_ln")
    logits = node(29, [wte, hf], "logits", [V, s], {}, "lm_head", storage=5)
    spec = {"name": name, "inputs": [ids, pids], "outputs": [logits],
            "parameters": sorted(params), "symbol_table": [s], "metadata": {},
            "tensors": tensors, "nodes": nodes}
    return spec, payload


# ------------------------------------------------------------------------------ GGUF writer

def _kv_str(key: str, val: str) -> bytes:
    k = key.encode()
    v = val.encode()
    return struct.pack("<Q", len(k)) + k + struct.pack("<I", 8) + struct.pack("<Q", len(v)) + v


def _kv_str_arr(key: str, vals: list[str]) -> bytes:
    k = key.encode()
    out = struct.pack("<Q", len(k)) + k + struct.pack("<I", 9) + struct.pack("<I", 8)
    out += struct.pack("<Q", len(vals))
    for v in vals:
        b = v.encode()
        out += struct.pack("<Q", len(b)) + b
    return out


def _nbytes(ne: list, ttype: int) -> int:
    n = int(np.prod(ne))
    return {Q8_0: n // 32 * 34, Q4_0: n // 32 * 18, F32: 4 * n, I32: 4 * n}[ttype]


def write_gguf(path: str | Path, spec: dict, payload: list[tuple], device: str | None = None) -> int:
    """Streams a GGUF v3 file (gguf.py:288-366 layout); returns bytes written."""
    kvs = [_kv_str("general.architecture", "ggmlc"), _kv_str("general.name", spec["name"]),
           _kv_str("ggmlc.version", "1.0.0"), _kv_str_arr("ggmlc.tasks", ["text-generation"]),
           _kv_str_arr("ggmlc.symbol_table", spec["symbol_table"]),
           _kv_str("ggmlc.graph_spec", json.dumps(spec, separators=(",", ":")))]
    infos = []
    off = 0
    for name, ne, ttype, _ in payload:
        shape = [int(v) if not isinstance(v, str) else 0 for v in ne]
        if ttype == I32 and any(isinstance(v, str) for v in ne):
            shape = [2048 if isinstance(v, str) else int(v) for v in ne]
        nb = _nbytes(shape, ttype)
        infos.append((name, shape, ttype, off, nb))
        off += (nb + ALIGN - 1) // ALIGN * ALIGN
    with open(path, "wb") as f:
        head = b"GGUF" + struct.pack("<I", 3) + struct.pack("<Q", len(infos)) + struct.pack("<Q", len(kvs))
        f.write(head)
        for kv in kvs:
            f.write(kv)
        for name, shape, ttype, o, _ in infos:
            b = name.encode()
            f.write(struct.pack("<Q", len(b)) + b + struct.pack("<I", len(shape)))
            for v in shape:
                f.write(struct.pack("<Q", v))
            f.write(struct.pack("<I", ttype) + struct.pack("<Q", o))
        pos = f.tell()
        pad = (ALIGN - pos % ALIGN) % ALIGN
        f.write(b"\0" * pad)
        data_start = f.tell()
        for (name, ne, ttype, maker), (_, shape, _, o, nb) in zip(payload, infos):
            assert f.tell() - data_start <= o
            f.write(b"\0" * (data_start + o - f.tell()))
            wrote = 0
            for chunk in maker(device):
                f.write(chunk.tobytes())
                wrote += chunk.size
            if wrote < nb:  # arange longer than requested max_seq is not needed: pad with zeros
                f.write(b"\0" * (nb - wrote))
            elif wrote > nb:
                raise ValueError(f"tensor {name}: payload {wrote} > {nb} bytes")
            f.write(b"\0" * ((ALIGN - (f.tell() - data_start) % ALIGN) % ALIGN))
        return f.tell()


def synth_llama(path: str | Path, shape: str | LlamaShape, qtype: int = Q4_0,
                device: str | None = None, name: str | None = None) -> Path:
    cfg = SHAPES[shape] if isinstance(shape, str) else shape
    spec, payload = llama_graph(cfg, qtype, name or (shape if isinstance(shape, str) else "llama"))
    write_gguf(path, spec, payload, device=device)
    return Path(path)


def synth_gpt2(path: str | Path, shape: str | GPT2Shape = "gpt2-small", qtype: int = Q8_0,
               device: str | None = None, name: str | None = None) -> Path:
    cfg = SHAPES[shape] if isinstance(shape, str) else shape
    spec, payload = gpt2_graph(cfg, qtype, name or (shape if isinstance(shape, str) else "gpt2"))
    write_gguf(path, spec, payload, device=device)
    return Path(path)


def synth_model(path: str | Path, shape: str, qtype: int, device: str | None = None,
                name: str | None = None) -> Path:
    """Either family by its SHAPES name."""
    if isinstance(SHAPES[shape], GPT2Shape):
        return synth_gpt2(path, shape, qtype, device, name)
    return synth_llama(path, shape, qtype, device, name)
