"""gb_attn_decode_noalloc: decode attention whose split scratch is a fixed static device array.

The GPU test calls it through the C ABI twice in a row (new tokens at kv_pos and kv_pos + 1) and
checks each call bit-for-bit against gb_attn_decode with a caller-allocated workspace, on
separate copies of the KV cache.  Caches of up to a few thousand positions run without split
scratch (thread-block clusters merge in distributed shared memory); the 8192-position case takes
the split path and so reads and writes the static array.  The file name sorts last so the test also runs after every
other test of a full session; it needs no state from them."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

import gpu_util as G
from conftest import cuda_available

P, I, I64, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float


def _lib():
    L = G.lib_fused()
    L.gb_attn_decode_noalloc.argtypes = [P, I64, I64, I64, P, P, I64, I64, I, F, P, I64, F, P,
                                         P, P, P]
    L.gb_attn_decode_noalloc_max_bytes.argtypes = []
    L.gb_attn_decode_noalloc_max_bytes.restype = ctypes.c_size_t
    return L


def test_noalloc_rejects_oversized_scratch():
    """A shape whose split partials exceed the static array fails with an error before any CUDA
    call, so this runs without a GPU."""
    L = _lib()
    assert L.gb_attn_decode_noalloc_max_bytes() == 4 << 20
    Hq, Hkv, hd, ctx = 64, 1, 256, 4096
    assert L.gb_attn_decode_workspace_bytes(Hq, Hkv, hd, ctx) > L.gb_attn_decode_noalloc_max_bytes()
    rc = L.gb_attn_decode_noalloc(None, Hq, Hkv, hd, None, None, ctx, 0, hd, 10000.0, None, 0,
                                  1.0, None, None, None, None)
    assert rc != 0
    assert "static array" in L.gb_last_error().decode()


@pytest.mark.gpu
@pytest.mark.skipif(not cuda_available(), reason="needs a CUDA device")
@pytest.mark.parametrize("Hq,Hkv,hd,ctx,kv_pos", [(32, 8, 128, 1024, 700), (4, 2, 64, 512, 0),
                                                   (64, 8, 128, 4096, 3000),
                                                   (32, 8, 128, 8192, 6000)])
def test_noalloc_matches_workspace_entry_point(Hq, Hkv, hd, ctx, kv_pos):
    torch = G.torch_dev()
    L = _lib()
    rng = np.random.default_rng(1000 + Hq + kv_pos)
    base = 500000.0
    n_pos = max(4096, ctx)
    tab = np.empty((n_pos, hd // 2, 2), np.float32)
    G.lib().gb_rope_table_fill(tab.ctypes.data, n_pos, hd, base)
    scale = float(np.float32(1.0) / np.sqrt(np.float32(hd)))
    assert L.gb_attn_decode_workspace_bytes(Hq, Hkv, hd, ctx) <= L.gb_attn_decode_noalloc_max_bytes()

    k0 = rng.standard_normal((Hkv, ctx, hd)).astype(np.float16).view(np.uint16)
    v0 = rng.standard_normal((Hkv, ctx, hd)).astype(np.float16).view(np.uint16)
    qkvs = [G.dev(rng.standard_normal((Hq + 2 * Hkv) * hd).astype(np.float32)) for _ in range(2)]
    t_d = G.dev(tab)
    # two independent caches: each entry point writes the new k/v rows into its own
    k_ref, v_ref, k_na, v_na = G.dev(k0), G.dev(v0), G.dev(k0), G.dev(v0)
    work = torch.empty(int(L.gb_attn_decode_workspace_bytes(Hq, Hkv, hd, ctx)), dtype=torch.uint8,
                       device="cuda")

    def outs():
        return (torch.full((Hq, hd), float("nan"), dtype=torch.float32, device="cuda"),
                torch.zeros(Hq * hd, dtype=torch.int8, device="cuda"),
                torch.full((Hq * hd // 32,), float("nan"), dtype=torch.float32, device="cuda"))

    o_ref = [outs() for _ in range(2)]
    o_na = [outs() for _ in range(2)]
    torch.cuda.synchronize()
    for step in range(2):
        pos = kv_pos + step
        o, oq, od = o_ref[step]
        G.check(L.gb_attn_decode(G.ptr(qkvs[step]), Hq, Hkv, hd, G.ptr(k_ref), G.ptr(v_ref), ctx,
                                 pos, hd, base, G.ptr(t_d), n_pos, scale, G.ptr(o), G.ptr(oq),
                                 G.ptr(od), G.ptr(work), None))
        o, oq, od = o_na[step]
        G.check(L.gb_attn_decode_noalloc(G.ptr(qkvs[step]), Hq, Hkv, hd, G.ptr(k_na), G.ptr(v_na),
                                         ctx, pos, hd, base, G.ptr(t_d), n_pos, scale, G.ptr(o),
                                         G.ptr(oq), G.ptr(od), None))
        torch.cuda.synchronize()
    # after the first (setup) call, calls leave the device's free memory untouched.  The reading
    # covers the whole device, so another process's allocation could move it: a window of eight
    # calls is taken up to three times and one unchanged window suffices (an allocation inside
    # the entry point would show in every window).
    o, oq, od = o_na[1]
    clean = False
    for _ in range(3):
        torch.cuda.synchronize()
        before = torch.cuda.mem_get_info()[0]
        for _ in range(8):
            G.check(L.gb_attn_decode_noalloc(G.ptr(qkvs[1]), Hq, Hkv, hd, G.ptr(k_na),
                                             G.ptr(v_na), ctx, kv_pos + 1, hd, base, G.ptr(t_d),
                                             n_pos, scale, G.ptr(o), G.ptr(oq), G.ptr(od), None))
        torch.cuda.synchronize()
        if torch.cuda.mem_get_info()[0] == before:
            clean = True
            break
    assert clean, "device free memory moved in every window of noalloc calls"

    for step in range(2):
        for a, b in zip(o_ref[step], o_na[step]):
            assert torch.equal(a, b), f"call {step}: outputs differ"
        assert not torch.isnan(o_na[step][0]).any()
    assert torch.equal(k_ref, k_na) and torch.equal(v_ref, v_na)
