"""CPU ORACLE — test infrastructure, not product code.

ctypes bindings for the C restatement in ``oracle/oracle.c`` plus a numpy walker that runs a
ggmlc-compiled GGUF decoder graph the way the reference CPU runtime does
(``runtime/src/executor.cpp``: ``prepare`` :1453, op lowering :1738-2810, padded-KV
``FLASH_ATTN_EXT`` :2091-2212).  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
CPU-baseline / reference legs may import this module, and only as the checker.

Parity: pinned against golden vectors produced by the reference itself (``oracle/_ref``, see
``tests/golden/make_golden.py``) in ``tests/test_oracle_golden.py``.
"""

from __future__ import annotations

import ctypes
import json
import os
import struct
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

F32, F16, Q4_0, Q8_0, I32, I64 = 0, 1, 2, 8, 26, 27
ATTN_MASK_MIN_FP16 = -32768.0  # runtime/include/ggmlc/types.h:240
KV_PAD = 256  # executor.h:181 kv_n_pad_


def build(force: bool = False) -> Path:
    """Compile oracle.c into oracle/liboracle.so (plain gcc, no contraction)."""
    src = HERE / "oracle.c"
    if force or not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        subprocess.check_call(
            ["gcc", "-O2", "-fPIC", "-shared", "-ffp-contract=off", "-o", str(LIB_PATH),
             str(src), "-lm"]
        )
    return LIB_PATH


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(str(LIB_PATH))
        P, I64_, F = ctypes.c_void_p, ctypes.c_int64, ctypes.c_float
        I = ctypes.c_int
        sig = {
            "oracle_fp32_to_fp16": ([F], ctypes.c_uint16),
            "oracle_fp16_to_fp32": ([ctypes.c_uint16], F),
            "oracle_dequantize_row": ([I, P, P, I64_], None),
            "oracle_quantize_row_q8_0": ([P, P, I64_], None),
            "oracle_quantize_row_q8_0_ref": ([P, P, I64_], None),
            "oracle_block_dot": ([I, P, P], ctypes.c_int32),
            "oracle_vec_dot": ([I, I64_, P, P], F),
            "oracle_mul_mat": ([I, P, I64_, I64_, P, I64_, P], None),
            "oracle_mul_mat_f32": ([P, I64_, I64_, P, I64_, P], None),
            "oracle_get_rows": ([I, P, I64_, P, I64_, P], None),
            "oracle_rms_norm": ([P, I64_, I64_, F, P, P], None),
            "oracle_layer_norm": ([P, I64_, I64_, F, P, P, P], None),
            "oracle_rope_neox": ([P, I64_, I64_, I64_, P, I, F, P], None),
            "oracle_swiglu": ([P, I64_, I64_, P], None),
            "oracle_bias_gelu": ([P, P, I64_, I64_, P], None),
            "oracle_flash_attn": ([P, P, P, P, I64_, I64_, I64_, I64_, I64_, F, P], None),
        }
        for name, (args, res) in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


# ----------------------------------------------------------------------------------- op level

def row_bytes(t: int, k: int) -> int:
    return {Q8_0: k // 32 * 34, Q4_0: k // 32 * 18, F16: 2 * k, F32: 4 * k}[t]


def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    """Rows of x (f32, last dim % 32 == 0) -> Q8_0 block bytes, AVX2 semantics."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    k = x.shape[-1]
    out = np.empty(x.shape[:-1] + (k // 32 * 34,), dtype=np.uint8)
    lib().oracle_quantize_row_q8_0(_p(x), _p(out), x.size)
    return out


def dequantize(t: int, data: np.ndarray, k: int) -> np.ndarray:
    data = np.ascontiguousarray(data, dtype=np.uint8)
    rows = data.size // row_bytes(t, k)
    out = np.empty((rows, k), dtype=np.float32)
    lib().oracle_dequantize_row(t, _p(data), _p(out), rows * k)
    return out


def mul_mat(wtype: int, w: np.ndarray, N: int, K: int, x: np.ndarray) -> np.ndarray:
    """Y[M,N] = X[M,K] . W^T, W in GGUF block rows (or f32 [N,K])."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, K)
    M = x.shape[0]
    y = np.empty((M, N), dtype=np.float32)
    if wtype == F32:
        w = np.ascontiguousarray(w, dtype=np.float32)
        lib().oracle_mul_mat_f32(_p(w), N, K, _p(x), M, _p(y))
    elif wtype == F16:
        wf = np.ascontiguousarray(np.frombuffer(w.tobytes(), np.float16).astype(np.float32))
        lib().oracle_mul_mat_f32(_p(wf), N, K, _p(x), M, _p(y))
    else:
        w = np.ascontiguousarray(w, dtype=np.uint8)
        lib().oracle_mul_mat(wtype, _p(w), N, K, _p(x), M, _p(y))
    return y


def rms_norm(x: np.ndarray, eps: float, gamma: np.ndarray | None = None) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    d = x.shape[-1]
    y = np.empty_like(x)
    g = None if gamma is None else np.ascontiguousarray(gamma, dtype=np.float32)
    lib().oracle_rms_norm(_p(x), d, x.size // d, eps, _p(g), _p(y))
    return y


def layer_norm(x, eps, gamma=None, beta=None):
    x = np.ascontiguousarray(x, dtype=np.float32)
    d = x.shape[-1]
    y = np.empty_like(x)
    g = None if gamma is None else np.ascontiguousarray(gamma, dtype=np.float32)
    b = None if beta is None else np.ascontiguousarray(beta, dtype=np.float32)
    lib().oracle_layer_norm(_p(x), d, x.size // d, eps, _p(g), _p(b), _p(y))
    return y


def rope_neox(x: np.ndarray, pos: np.ndarray, n_dims: int, freq_base: float) -> np.ndarray:
    """x: [s, H, hd] f32, pos: [s] int32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    s, H, hd = x.shape
    pos = np.ascontiguousarray(pos, dtype=np.int32)
    y = np.empty_like(x)
    lib().oracle_rope_neox(_p(x), hd, H, s, _p(pos), n_dims, freq_base, _p(y))
    return y


def swiglu(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    ffn = x.shape[-1] // 2
    y = np.empty(x.shape[:-1] + (ffn,), dtype=np.float32)
    lib().oracle_swiglu(_p(x), ffn, x.size // (2 * ffn), _p(y))
    return y


def bias_gelu(x: np.ndarray, b: np.ndarray | None) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    d = x.shape[-1]
    y = np.empty_like(x)
    bb = None if b is None else np.ascontiguousarray(b, dtype=np.float32).reshape(-1)
    lib().oracle_bias_gelu(_p(x), _p(bb), d, x.size // d, _p(y))
    return y


def flash_attn(q, k16, v16, mask16, scale):
    """q [s,Hq,hd] f32; k16/v16 [Hkv,n_kv,hd] uint16 (f16 bits); mask16 [s,n_kv] or None."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    s, Hq, hd = q.shape
    Hkv, n_kv, _ = k16.shape
    k16 = np.ascontiguousarray(k16, dtype=np.uint16)
    v16 = np.ascontiguousarray(v16, dtype=np.uint16)
    m = None if mask16 is None else np.ascontiguousarray(mask16, dtype=np.uint16)
    y = np.empty_like(q)
    lib().oracle_flash_attn(_p(q), _p(k16), _p(v16), _p(m), hd, s, Hq, Hkv, n_kv, scale, _p(y))
    return y


def causal_mask_f16(pos: int, s: int, n_kv: int) -> np.ndarray:
    """fill_f16_causal_mask (executor.cpp:136-148)."""
    j = np.arange(n_kv)[None, :]
    i = np.arange(s)[:, None]
    m = np.where(j <= pos + i, 0.0, ATTN_MASK_MIN_FP16).astype(np.float16)
    return m.view(np.uint16)


def pad_kv_len(n_kv: int, max_ctx: int, n_pad: int = KV_PAD) -> int:
    """pad_kv_len (executor.cpp:58-64)."""
    n_kv = max(n_kv, 1)
    if n_pad <= 1:
        return min(n_kv, max_ctx)
    padded = max(n_pad, (n_kv + n_pad - 1) // n_pad * n_pad)
    return min(padded, max_ctx)


# ------------------------------------------------------------------------------------- GGUF

_GGUF_SCALAR = {0: "B", 1: "b", 2: "H", 3: "h", 4: "I", 5: "i", 6: "f", 7: "?", 10: "Q", 11: "q",
                12: "d"}


def read_gguf(path_or_bytes) -> tuple[dict, dict, dict]:
    """Minimal GGUF v3 reader: (kv, tensor_infos{name: (dims, type, offset)}, data_by_name)."""
    buf = Path(path_or_bytes).read_bytes() if not isinstance(path_or_bytes, (bytes, bytearray)) \
        else bytes(path_or_bytes)
    off = 0

    def rd(fmt):
        nonlocal off
        v = struct.unpack_from("<" + fmt, buf, off)
        off += struct.calcsize("<" + fmt)
        return v[0] if len(v) == 1 else v

    def rstr():
        nonlocal off
        n = rd("Q")
        s = buf[off:off + n].decode("utf-8")
        off += n
        return s

    def rval(t):
        if t == 8:
            return rstr()
        if t == 9:
            et = rd("I")
            n = rd("Q")
            return [rval(et) for _ in range(n)]
        return rd(_GGUF_SCALAR[t])

    if buf[:4] != b"GGUF":
        raise ValueError("not a GGUF file")
    off = 4
    rd("I")
    nt = rd("Q")
    nkv = rd("Q")
    kv = {}
    for _ in range(nkv):
        k = rstr()
        kv[k] = rval(rd("I"))
    infos = {}
    for _ in range(nt):
        name = rstr()
        nd = rd("I")
        dims = [rd("Q") for _ in range(nd)]
        t = rd("I")
        o = rd("Q")
        infos[name] = (dims, t, o)
    align = int(kv.get("general.alignment", 32))
    data_off = (off + align - 1) // align * align
    data = {}
    for name, (dims, t, o) in infos.items():
        n = int(np.prod(dims))
        nbytes = {F32: 4 * n, F16: 2 * n, Q8_0: n // 32 * 34, Q4_0: n // 32 * 18, I32: 4 * n,
                  I64: 8 * n, 24: n, 25: 2 * n, 28: 8 * n}[t]
        data[name] = np.frombuffer(buf, dtype=np.uint8, count=nbytes, offset=data_off + o)
    return kv, infos, data


# ------------------------------------------------------------------------------ graph walker

def _eval_dim(d: dict, env: dict) -> int:
    t = d.get("type", "static")
    if t == "static":
        return int(d.get("val", 1))
    if t == "symbol":
        return int(env[d["name"]])
    a, b = _eval_dim(d["left"], env), _eval_dim(d["right"], env)
    return {"add": a + b, "sub": a - b, "mul": a * b, "floordiv": a // b,
            "ceildiv": (a + b - 1) // b}[t]


class ModelOracle:
    """Runs a ggmlc GGUF decoder graph on the CPU with the oracle ops.

    Mirrors the reference executor: with ``init_kv_cache`` the attention K/V are written (F16)
    into a per-op cache at rows pos..pos+s-1 and attention runs over the padded window
    ``pad_kv_len(pos+s)`` with the F16 causal mask; without it, attention runs over the call's
    own K/V with a causal mask.  Arrays are kept in numpy order (ggml ne reversed).
    """

    def __init__(self, path_or_bytes):
        kv, infos, data = read_gguf(path_or_bytes)
        self.spec = json.loads(kv["ggmlc.graph_spec"])
        self.tensors = {int(k): v for k, v in self.spec["tensors"].items()}
        self.nodes = self.spec["nodes"]
        self.inputs = list(self.spec["inputs"])
        self.outputs = list(self.spec["outputs"])
        self.symbols = list(self.spec["symbol_table"])
        self.data = {}
        for tid, t in self.tensors.items():
            if t["name"] in data:
                self.data[tid] = data[t["name"]]
        self.kv_max_ctx = 0
        self.k_cache: dict[int, np.ndarray] = {}
        self.v_cache: dict[int, np.ndarray] = {}
        self.logits_last_only = False

    # KV enable rule of init_kv_cache (executor.cpp:505-539)
    def init_kv_cache(self, max_ctx: int = 2048) -> bool:
        has_rope = any(n["opcode"] == 48 for n in self.nodes)
        has_pos_in = any("pos" in self.tensors[i]["name"] for i in self.inputs)
        has_arange = any("arange" in t["name"] and tid in self.data
                         for tid, t in self.tensors.items())
        if not (has_rope or has_pos_in or has_arange or "pos" in self.symbols):
            return False
        self.kv_max_ctx = max_ctx
        self.k_cache.clear()
        self.v_cache.clear()
        return True

    def reset_kv_cache(self):
        for c in list(self.k_cache.values()) + list(self.v_cache.values()):
            c[...] = 0

    def _shape(self, tid, env):
        ne = [_eval_dim(d, env) for d in self.tensors[tid]["ne"]]
        return ne

    def _np_shape(self, ne):
        return (ne[3], ne[2], ne[1], ne[0])

    def _param(self, tid, env):
        t = self.tensors[tid]
        raw = self.data[tid]
        ty = t["type"]
        ne = self._shape(tid, env)
        if ty == F32:
            return np.frombuffer(raw.tobytes(), np.float32)[: int(np.prod(ne))].reshape(
                self._np_shape(ne))
        if ty == I32:
            return np.frombuffer(raw.tobytes(), np.int32)
        return raw  # quantized / f16 bytes, interpreted by the consumer

    def forward(self, tokens: np.ndarray, pos: int | None = None,
                position_ids: np.ndarray | None = None) -> np.ndarray:
        tokens = np.asarray(tokens, dtype=np.int32).reshape(-1)
        s = tokens.size
        env = {sym: s for sym in self.symbols}
        env["s"] = s
        use_kv = pos is not None and self.kv_max_ctx > 0
        p0 = pos if pos is not None else 0
        vals: dict[int, np.ndarray] = {}
        vals[self.inputs[0]] = tokens.reshape(1, 1, 1, s)
        if len(self.inputs) > 1:
            pid = position_ids if position_ids is not None else np.arange(p0, p0 + s)
            vals[self.inputs[1]] = np.asarray(pid, np.int32).reshape(1, 1, 1, s)

        def get(tid):
            if tid in vals:
                return vals[tid]
            t = self.tensors[tid]
            if tid in self.data:
                if t["type"] == I32 and "arange" in t["name"]:
                    a = np.frombuffer(self.data[tid].tobytes(), np.int32)
                    off = p0 if use_kv else 0
                    return a[off:off + s].reshape(1, 1, 1, s)
                return self._param(tid, env)
            raise KeyError(f"tensor {tid} ({t['name']}) has no value")

        for node in self.nodes:
            op = node["opcode"]
            ins = node["inputs"]
            out = node["outputs"][0]
            attrs = node.get("attributes", {})
            one = self._shape(out, env)
            if op == 40:  # GET_ROWS
                w = self.tensors[ins[0]]
                d = self._shape(ins[0], env)[0]
                ids = np.asarray(get(ins[1]), np.int32).reshape(-1)
                rows = np.empty((ids.size, d), np.float32)
                raw = np.ascontiguousarray(self.data[ins[0]])
                lib().oracle_get_rows(w["type"], _p(raw), d, _p(ids), ids.size, _p(rows))
                vals[out] = rows.reshape(self._np_shape(one))
            elif op in (202, 25):  # RMS_NORM (+ gamma)
                x = get(ins[0])
                g = get(ins[1]).reshape(-1) if len(ins) > 1 else None
                vals[out] = rms_norm(x, float(attrs.get("eps", 1e-5)), g)
            elif op in (201, 24):  # LayerNorm (+ gamma, beta)
                x = get(ins[0])
                g = get(ins[1]).reshape(-1) if len(ins) > 1 else None
                b = get(ins[2]).reshape(-1) if len(ins) > 2 else None
                vals[out] = layer_norm(x, float(attrs.get("eps", 1e-5)), g, b)
            elif op == 29:  # MUL_MAT (+ bias)
                wt = self.tensors[ins[0]]
                K, N = self._shape(ins[0], env)[:2]
                x = get(ins[1])
                lead = x.shape[:-1]
                xr = np.ascontiguousarray(x).reshape(-1, K)
                if self.logits_last_only and out in self.outputs and xr.shape[0] > 1:
                    xr = xr[-1:]
                    lead = (1, 1, 1)
                y = mul_mat(wt["type"], self.data[ins[0]], N, K, xr)
                if len(ins) > 2:
                    y = y + get(ins[2]).reshape(-1)[None, :]
                vals[out] = y.reshape(lead + (N,))
            elif op == 37:  # VIEW / slice
                x = get(ins[0])
                gd = int(attrs.get("ggml_dim", 0))
                ax = 3 - gd
                sl = [slice(None)] * 4
                sl[ax] = slice(int(attrs["start"]), int(attrs["end"]), int(attrs.get("step", 1)))
                vals[out] = x[tuple(sl)]
            elif op == 36:  # RESHAPE
                vals[out] = np.ascontiguousarray(get(ins[0])).reshape(self._np_shape(one))
            elif op in (38, 39):  # PERMUTE / TRANSPOSE
                x = get(ins[0])
                axes = [int(attrs.get(f"axis{i}", i)) for i in range(4)]
                perm = [0] * 4
                for i in range(4):
                    perm[3 - axes[i]] = 3 - i
                vals[out] = np.transpose(x, perm)
            elif op == 48:  # ROPE (NEOX)
                x = get(ins[0])  # numpy (1, s, H, hd)
                pos_arr = np.asarray(get(ins[1]), np.int32).reshape(-1)
                n_dims = int(attrs.get("n_dims", x.shape[-1]))
                fb = float(attrs.get("freq_base", 10000.0))
                xs = np.ascontiguousarray(x).reshape(x.shape[-3], x.shape[-2], x.shape[-1])
                vals[out] = rope_neox(xs, pos_arr, n_dims, np.float32(fb)).reshape(x.shape)
            elif op == 74:  # FLASH_ATTN_EXT
                vals[out] = self._attn(node, get, env, use_kv, p0)
            elif op == 2:  # ADD
                vals[out] = (get(ins[0]) + get(ins[1])).astype(np.float32)
            elif op == 7:  # MUL
                vals[out] = (get(ins[0]) * get(ins[1])).astype(np.float32)
            elif op in (203, 100):  # SWIGLU on concatenated [gate; up]
                vals[out] = swiglu(get(ins[0]))
            elif op == 200:  # bias + GELU
                b = get(ins[1]) if len(ins) > 1 else None
                vals[out] = bias_gelu(get(ins[0]), b)
            else:
                raise NotImplementedError(f"oracle: opcode {op} ({node.get('name')})")
        return np.ascontiguousarray(vals[self.outputs[0]], dtype=np.float32)

    def _attn(self, node, get, env, use_kv, p0):
        ins = node["inputs"]
        attrs = node.get("attributes", {})
        q = get(ins[0])  # numpy (1, Hq, s, hd)
        k = get(ins[1])  # (1, Hkv, s, hd)
        v = get(ins[2])
        _, Hq, s, hd = q.shape
        Hkv = k.shape[1]
        scale = float(attrs.get("scale", 1.0 / np.sqrt(np.float32(hd))))
        scale = float(np.float32(1.0) / np.sqrt(np.float32(hd))) if "scale" not in attrs else scale
        qs = np.ascontiguousarray(np.transpose(q[0], (1, 0, 2)))  # [s, Hq, hd]
        k16 = np.ascontiguousarray(k[0]).astype(np.float16).view(np.uint16)
        v16 = np.ascontiguousarray(v[0]).astype(np.float16).view(np.uint16)
        if use_kv:
            oid = node["id"]
            if oid not in self.k_cache:
                self.k_cache[oid] = np.zeros((Hkv, self.kv_max_ctx, hd), np.uint16)
                self.v_cache[oid] = np.zeros((Hkv, self.kv_max_ctx, hd), np.uint16)
            kc, vc = self.k_cache[oid], self.v_cache[oid]
            kc[:, p0:p0 + s, :] = k16
            vc[:, p0:p0 + s, :] = v16
            n_kv = pad_kv_len(p0 + s, self.kv_max_ctx)
            mask = causal_mask_f16(p0, s, n_kv)
            y = flash_attn(qs, kc[:, :n_kv], vc[:, :n_kv], mask, scale)
        else:
            mask = causal_mask_f16(0, s, s) if (attrs.get("is_causal", 0) and s > 1) else None
            y = flash_attn(qs, k16, v16, mask, scale)
        # y: [s, Hq, hd] == ggml ne [hd, Hq, s] (fused_transpose result)
        if attrs.get("fused_transpose", 0):
            return y.reshape(1, s, Hq, hd)
        return np.transpose(y, (1, 0, 2)).reshape(1, Hq, s, hd)
