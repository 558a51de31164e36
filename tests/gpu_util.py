"""Helpers for the GPU tests: device buffers (torch, as plumbing), typed bindings of the
op-level C ABI entry points, and random valid GGUF weight blocks."""

from __future__ import annotations

import ctypes

import numpy as np

from oracle import oracle as O


def torch_dev():
    import torch

    return torch


def dev(a: np.ndarray):
    torch = torch_dev()
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def ptr(t) -> int:
    return 0 if t is None else int(t.data_ptr())


def lib():
    from ggmlc_b200 import _runtime

    L = _runtime.lib()
    P, I, I64, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
    L.gb_repack_blocks.argtypes = [P, I, I64, I64, P, P]
    L.gb_weight_row_bytes.argtypes = [I, I64]
    L.gb_weight_row_bytes.restype = I64
    L.gb_quantize_q8_0.argtypes = [P, I64, I64, I64, P, P, P]
    L.gb_mul_mat_q.argtypes = [I, P, I64, I64, P, P, I64, P, P, P, P]
    L.gb_gemm_tc.argtypes = [I, P, I64, I64, P, P, I64, P, P, P, P]
    L.gb_get_rows.argtypes = [I, P, I64, I64, P, I64, P, P]
    L.gb_rms_norm.argtypes = [P, I64, I64, F, P, P, P, P, P]
    L.gb_swiglu.argtypes = [P, I64, I64, P, P, P, P]
    L.gb_layer_norm.argtypes = [P, I64, I64, F, P, P, P, P, P, P]
    L.gb_bias_gelu.argtypes = [P, P, I64, I64, P, P, P, P]
    L.gb_rope_table_fill.argtypes = [P, I64, I, F]
    L.gb_rope_table_fill.restype = F
    L.gb_rope_neox.argtypes = [P, I64, I64, I64, P, I, F, P, I64, P, P]
    L.gb_attention_workspace_bytes.argtypes = [I64, I64, I64, I64]
    L.gb_attention_workspace_bytes.restype = ctypes.c_size_t
    L.gb_attention.argtypes = [P, P, P, I64, I64, I64, I64, I64, I64, F, P, P, P]
    return L


def check(rc: int):
    if rc != 0:
        from ggmlc_b200 import _runtime

        raise RuntimeError(_runtime.lib().gb_last_error().decode())


def random_blocks(rng, wtype: int, N: int, K: int, scale: float = 0.01) -> np.ndarray:
    """N rows of K elements as GGUF block bytes with valid quants and N(0, scale) fp16 scales."""
    bb = 34 if wtype == O.Q8_0 else 18
    nb = K // 32
    w = rng.integers(0, 256, size=(N, nb, bb), dtype=np.uint8)
    if wtype == O.Q8_0:
        q = w[:, :, 2:]
        q[q == 128] = 129
    d = (rng.standard_normal((N, nb)) * scale).astype(np.float16)
    w[:, :, 0:2] = d.view(np.uint8).reshape(N, nb, 2)
    return w.reshape(N, nb * bb)


def upload_weight(wtype: int, blocks: np.ndarray, N: int, K: int):
    """GGUF block bytes -> device weight in the split-row layout (gb_repack_blocks)."""
    torch = torch_dev()
    src = dev(blocks.reshape(-1))
    rb = lib().gb_weight_row_bytes(wtype, K)
    assert rb > 0
    wq = torch.empty(N * rb, dtype=torch.uint8, device="cuda")
    check(lib().gb_repack_blocks(ptr(src), wtype, N, K, ptr(wq), None))
    torch.cuda.synchronize()
    return wq, None


def quantize(x_dev, M: int, K: int):
    torch = torch_dev()
    xq = torch.empty((M, K), dtype=torch.int8, device="cuda")
    xd = torch.empty((M, K // 32), dtype=torch.float32, device="cuda")
    check(lib().gb_quantize_q8_0(ptr(x_dev), K, M, K, ptr(xq), ptr(xd), None))
    return xq, xd


def mul_mat(wtype, wq, wd, N, K, x_dev, M, bias=None, residual=None, tc=False):
    """gb_mul_mat_q (the dispatching entry), or with tc=True the tensor-core GEMM gb_gemm_tc."""
    torch = torch_dev()
    xq, xd = quantize(x_dev, M, K)
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    fn = lib().gb_gemm_tc if tc else lib().gb_mul_mat_q
    check(fn(wtype, ptr(wq), N, K, ptr(xq), ptr(xd), M, ptr(y), ptr(bias), ptr(residual), None))
    torch.cuda.synchronize()
    return y.cpu().numpy()


def lib_fused():
    L = lib()
    P, I, I64, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
    L.gb_gemv.argtypes = [I, P, I64, I64, I64, P, P, P, F, P, I, P, P, P, P, P, P]
    L.gb_attn_decode_workspace_bytes.argtypes = [I64, I64, I64, I64]
    L.gb_attn_decode_workspace_bytes.restype = ctypes.c_size_t
    L.gb_attn_decode.argtypes = [P, I64, I64, I64, P, P, I64, I64, I, F, P, I64, F, P, P, P, P, P]
    return L
