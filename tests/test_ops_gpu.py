"""Operator parity on the GPU: each kernel called through the C ABI (include/ggmlc_b200.h)
against the CPU oracle (pinned bit-exact to the reference) on the same seeded inputs.

Bars: bit-exact for quantization, dequantization, decode matmul (M <= 8, which reproduces the
CPU's fp32 lane order), RMSNorm, RoPE and SwiGLU; the prefill matmul (M > 8, int8 tensor-core
block sums) within 1e-5 of max|y| (north star: 1e-3 relative); attention (fp32 accumulation vs
the CPU's fp16 accumulator) within 2e-3 of max|y|."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import cuda_available
from oracle import oracle as O

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not cuda_available(), reason="needs a CUDA device")]


@pytest.fixture(scope="module")
def G():
    import gpu_util

    return gpu_util


def _x(rng, M, K, ties=True):
    x = rng.standard_normal((M, K)).astype(np.float32)
    if ties and M > 1:
        # exact .5 ties of x*127/amax in the first block of row 0
        x[0, 0] = 127.0
        x[0, 1:32] = np.arange(31, dtype=np.float32) + 0.5
    x[-1, 32:64] = 0.0  # an all-zero block (amax = 0)
    return x


@pytest.mark.parametrize("M,K", [(1, 32), (3, 256), (17, 4096), (64, 14336)])
def test_quantize_bit_exact(G, M, K):
    rng = np.random.default_rng(M * 7 + K)
    x = _x(rng, M, K)
    xq, xd = G.quantize(G.dev(x), M, K)
    ref = O.quantize_q8_0(x).reshape(M, K // 32, 34)
    ref_q = ref[:, :, 2:].reshape(M, K).view(np.int8)
    ref_d = ref[:, :, :2].copy().view(np.float16).reshape(M, K // 32).astype(np.float32)
    assert np.array_equal(xq.cpu().numpy(), ref_q)
    assert np.array_equal(xd.cpu().numpy(), ref_d)


def _close(y, ref, rel=1e-5):
    """fp32 block accumulation order differs from the CPU lanes: compare to the output range."""
    return np.max(np.abs(y - ref)) <= rel * max(np.max(np.abs(ref)), 1e-30)


def _int_exact_case(rng, wtype, N, K, M):
    """Weights with one power-of-two scale per row and activations whose Q8_0 scale is exactly 1
    (one element of 127 per block, the rest in [-3, 3]): every block term and every partial sum
    is an exactly representable fp32 value (|sum| < 2^24 grid steps even at K = 14336), so any
    summation order gives the same result and the GPU must reproduce the oracle bit for bit —
    this pins the integer block dots."""
    w = _pow2_blocks(rng, wtype, N, K)
    x = rng.integers(-3, 4, size=(M, K)).astype(np.float32)
    x[:, ::32] = 127.0
    return w, x


def _pow2_blocks(rng, wtype, N, K):
    bb = 34 if wtype == O.Q8_0 else 18
    nb = K // 32
    w = rng.integers(0, 256, size=(N, nb, bb), dtype=np.uint8)
    if wtype == O.Q8_0:
        q = w[:, :, 2:]
        q[q == 128] = 129
    # one power-of-two scale per row keeps every partial sum on a 2^e grid below 2^24 steps
    d = np.broadcast_to(2.0 ** rng.integers(-12, -6, size=(N, 1)), (N, nb)).astype(np.float16)
    w[:, :, 0:2] = d.view(np.uint8).reshape(N, nb, 2)
    return w.reshape(N, nb * bb)


@pytest.mark.parametrize("wtype", [O.Q8_0, O.Q4_0])
@pytest.mark.parametrize("M", [1, 2, 5, 8, 12, 16])
@pytest.mark.parametrize("N,K", [(64, 256), (300, 4096), (40, 14336), (50, 576)])
def test_decode_matmul_close(G, wtype, M, N, K):
    rng = np.random.default_rng(N + K + M + wtype)
    w = G.random_blocks(rng, wtype, N, K)
    wq, wd = G.upload_weight(wtype, w, N, K)
    x = _x(rng, M, K)
    y = G.mul_mat(wtype, wq, wd, N, K, G.dev(x), M)
    assert _close(y, O.mul_mat(wtype, w, N, K, x))


@pytest.mark.parametrize("path", ["default", "mma", "tc"])
@pytest.mark.parametrize("wtype", [O.Q8_0, O.Q4_0])
@pytest.mark.parametrize("M,N,K", [(1, 300, 4096), (3, 77, 14336), (8, 64, 576), (16, 96, 1024),
                                   (11, 100, 576), (17, 40, 1024), (64, 40, 4096)])
def test_matmul_integer_path_bit_exact(G, wtype, M, N, K, path, monkeypatch):
    """Decode (M <= 16) and prefill (M > 16) kernels on inputs where fp32 summation is exact;
    prefill on the routed GEMM path and on each path forced by GGMLC_B200_GEMM."""
    if path != "default":
        if M <= 16:
            pytest.skip("decode rows do not use the prefill GEMM")
        monkeypatch.setenv("GGMLC_B200_GEMM", path)
    rng = np.random.default_rng(7 * N + K + M + wtype)
    w, x = _int_exact_case(rng, wtype, N, K, M)
    wq, wd = G.upload_weight(wtype, w, N, K)
    y = G.mul_mat(wtype, wq, wd, N, K, G.dev(x), M)
    assert np.array_equal(y, O.mul_mat(wtype, w, N, K, x))


@pytest.mark.parametrize("wtype", [O.Q8_0, O.Q4_0])
def test_decode_matmul_epilogue(G, wtype):
    rng = np.random.default_rng(5)
    N, K, M = 96, 512, 3
    w, x = _int_exact_case(rng, wtype, N, K, M)
    wq, wd = G.upload_weight(wtype, w, N, K)
    bias = rng.standard_normal(N).astype(np.float32)
    res = rng.standard_normal((M, N)).astype(np.float32)
    y = G.mul_mat(wtype, wq, wd, N, K, G.dev(x), M, bias=G.dev(bias), residual=G.dev(res))
    ref = O.mul_mat(wtype, w, N, K, x)
    ref = res + (ref + bias[None, :]).astype(np.float32)
    assert np.array_equal(y, ref.astype(np.float32))


@pytest.mark.parametrize("path", ["default", "mma", "tc"])
@pytest.mark.parametrize("wtype", [O.Q8_0, O.Q4_0])
@pytest.mark.parametrize("M", [17, 64, 130])
def test_prefill_gemm_swiglu_epilogue(G, wtype, M, path, monkeypatch):
    """Prefill gate_up GEMM with SwiGLU and Q8_0 quantization fused in its epilogue (a tile of
    64 gate rows + the 64 matching up rows): bit-exact with the CPU SwiGLU and quantizer applied
    to the plain GEMM's outputs, on the routed path and on each path forced by GGMLC_B200_GEMM."""
    if path != "default":
        monkeypatch.setenv("GGMLC_B200_GEMM", path)
    torch = G.torch_dev()
    rng = np.random.default_rng(M + 100 * wtype)
    F, K = 192, 1024
    N = 2 * F
    w = G.random_blocks(rng, wtype, N, K, scale=0.05)
    wq, wd = G.upload_weight(wtype, w, N, K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    xq, xd = G.quantize(G.dev(x), M, K)
    y = torch.empty((M, F), dtype=torch.float32, device="cuda")
    yq = torch.empty((M, F), dtype=torch.int8, device="cuda")
    yd = torch.empty((M, F // 32), dtype=torch.float32, device="cuda")
    L = G.lib_fused()
    G.check(L.gb_gemv(wtype, G.ptr(wq), N, K, M, G.ptr(xq), G.ptr(xd), None, 0.0, None, 1,
                      G.ptr(y), G.ptr(yq), G.ptr(yd), None, None, None))
    gu = torch.empty((M, N), dtype=torch.float32, device="cuda")
    G.check(L.gb_mul_mat_q(wtype, G.ptr(wq), N, K, G.ptr(xq), G.ptr(xd), M, G.ptr(gu), None, None,
                           None))
    h = O.swiglu(gu.cpu().numpy())
    assert np.array_equal(y.cpu().numpy(), h)
    hq = O.quantize_q8_0(h).reshape(M, F // 32, 34)
    assert np.array_equal(yq.cpu().numpy(), hq[:, :, 2:].reshape(M, F).view(np.int8))
    assert np.array_equal(yd.cpu().numpy(),
                          hq[:, :, :2].copy().view(np.float16).reshape(M, F // 32).astype(np.float32))


@pytest.mark.parametrize("wtype", [O.Q8_0, O.Q4_0])
@pytest.mark.parametrize("M", [200, 600])
def test_prefill_gemm_tile_variants(G, wtype, M):
    """Prefill shapes on both builds of the mma.sync block GEMM, which serves K % 128 != 0 (Q4_0
    at 600 rows has tiles for two CTAs per SM and runs the rolled build; 200 rows and Q8_0 run
    one CTA per SM): the integer path is
    bit-exact against the oracle on sampled output columns, and the SwiGLU epilogue is bit-exact
    against the plain GEMM's outputs."""
    torch = G.torch_dev()
    rng = np.random.default_rng(M + 7 * wtype)
    F, K = 4096, 288  # K % 128 != 0: the mma.sync block GEMM (the tcgen05 GEMM takes the rest)
    N = 2 * F
    w, x = _int_exact_case(rng, wtype, N, K, M)
    wq, wd = G.upload_weight(wtype, w, N, K)
    y = G.mul_mat(wtype, wq, wd, N, K, G.dev(x), M)
    cols = np.sort(rng.choice(N, size=64, replace=False))
    assert np.array_equal(y[:, cols], O.mul_mat(wtype, np.ascontiguousarray(w[cols]), len(cols), K, x))
    xq, xd = G.quantize(G.dev(x), M, K)
    h = torch.empty((M, F), dtype=torch.float32, device="cuda")
    hq = torch.empty((M, F), dtype=torch.int8, device="cuda")
    hd = torch.empty((M, F // 32), dtype=torch.float32, device="cuda")
    L = G.lib_fused()
    G.check(L.gb_gemv(wtype, G.ptr(wq), N, K, M, G.ptr(xq), G.ptr(xd), None, 0.0, None, 1,
                      G.ptr(h), G.ptr(hq), G.ptr(hd), None, None, None))
    ref = O.swiglu(y)
    assert np.array_equal(h.cpu().numpy(), ref)
    rq = O.quantize_q8_0(ref).reshape(M, F // 32, 34)
    assert np.array_equal(hq.cpu().numpy(), rq[:, :, 2:].reshape(M, F).view(np.int8))
    del wq, wd
    torch.cuda.empty_cache()


@pytest.mark.parametrize("wtype", [O.Q8_0, O.Q4_0])
@pytest.mark.parametrize("K", [576, 4096, 14336])
def test_decode_rows_independent_of_batch(G, wtype, K):
    """A row's decode-matmul result is bit-identical whatever rows run with it, with the
    residual and with the SwiGLU epilogue, within each decode kernel: the GEMV (1-2 rows) and
    the tensor-core kernel (3-16 rows).  Continuous batching thus returns a sequence's own
    logits whatever batch of the same kernel it joins."""
    torch = G.torch_dev()
    rng = np.random.default_rng(K + wtype)
    F = 96
    N = 2 * F
    w = G.random_blocks(rng, wtype, N, K, scale=0.05)
    wq, wd = G.upload_weight(wtype, w, N, K)
    x = rng.standard_normal((16, K)).astype(np.float32)
    res = rng.standard_normal((16, N)).astype(np.float32)
    xq, xd = G.quantize(G.dev(x), 16, K)
    res_d = G.dev(res)
    L = G.lib_fused()

    def run(rows):
        M = len(rows)
        q = xq[rows].contiguous()
        d = xd[rows].contiguous()
        r = res_d[rows].contiguous()
        y = torch.empty((M, N), dtype=torch.float32, device="cuda")
        G.check(L.gb_gemv(wtype, G.ptr(wq), N, K, M, G.ptr(q), G.ptr(d), None, 0.0, None, 0,
                          G.ptr(y), None, None, None, G.ptr(r), None))
        h = torch.empty((M, F), dtype=torch.float32, device="cuda")
        hq = torch.empty((M, F), dtype=torch.int8, device="cuda")
        hd = torch.empty((M, F // 32), dtype=torch.float32, device="cuda")
        G.check(L.gb_gemv(wtype, G.ptr(wq), N, K, M, G.ptr(q), G.ptr(d), None, 0.0, None, 1,
                          G.ptr(h), G.ptr(hq), G.ptr(hd), None, None, None))
        return y, h, hq, hd

    def check(base, sizes):
        for M in sizes:
            rows = list(range(16 - M, 16))
            outs = run(rows)
            for i, r in enumerate(rows):
                for got, ref in zip(outs, base[r]):
                    assert torch.equal(got[i], ref), f"M={M} row {r}"

    alone = [tuple(t[0] for t in run([r])) for r in range(16)]
    check(alone, (2,))
    by8 = [None] * 16
    for b in range(2):
        outs = run(list(range(8 * b, 8 * b + 8)))
        for i in range(8):
            by8[8 * b + i] = tuple(t[i] for t in outs)
    check(by8, (3, 4, 5, 11, 16))
    ref = O.mul_mat(wtype, w, N, K, x)
    for base in (alone, by8):
        got = np.stack([b[0].cpu().numpy() for b in base]) - res
        assert _close(got, ref)


@pytest.mark.parametrize("wtype", [O.Q8_0, O.Q4_0])
@pytest.mark.parametrize("M,N,K", [(17, 64, 256), (64, 200, 1024), (130, 77, 4096)])
def test_prefill_matmul_close(G, wtype, M, N, K):
    rng = np.random.default_rng(M * N + K)
    w = G.random_blocks(rng, wtype, N, K)
    wq, wd = G.upload_weight(wtype, w, N, K)
    x = _x(rng, M, K)
    y = G.mul_mat(wtype, wq, wd, N, K, G.dev(x), M)
    ref = O.mul_mat(wtype, w, N, K, x)
    assert np.max(np.abs(y - ref)) <= 1e-5 * np.max(np.abs(ref))


@pytest.mark.parametrize("wtype", [O.Q8_0, O.Q4_0])
@pytest.mark.parametrize("M,N,K", [(17, 40, 1024), (64, 300, 640), (130, 77, 4096),
                                   (300, 256, 2048), (5, 128, 14336), (600, 1000, 4096)])
def test_tensor_core_gemm_integer_path_bit_exact(G, wtype, M, N, K):
    """tcgen05 GEMM (gb_gemm_tc): partial row / column tiles, a partial 64-block scale group
    (K = 640), long K, M below one tile and several activation tiles, on inputs where fp32
    summation is exact."""
    rng = np.random.default_rng(11 * N + K + M + wtype)
    w, x = _int_exact_case(rng, wtype, N, K, M)
    wq, wd = G.upload_weight(wtype, w, N, K)
    y = G.mul_mat(wtype, wq, wd, N, K, G.dev(x), M, tc=True)
    assert G.lib().gb_gemm_tc_error() == 0
    assert np.array_equal(y, O.mul_mat(wtype, w, N, K, x))


@pytest.mark.parametrize("wtype", [O.Q8_0, O.Q4_0])
@pytest.mark.parametrize("M,N,K", [(64, 200, 1024), (512, 384, 4096)])
def test_tensor_core_gemm_close_with_epilogue(G, wtype, M, N, K):
    """tcgen05 GEMM on random data, with bias and residual, within 1e-5 of the output range of
    the oracle and equal to the dispatching entry wherever that runs the same block order."""
    rng = np.random.default_rng(M + N + K)
    w = G.random_blocks(rng, wtype, N, K)
    wq, wd = G.upload_weight(wtype, w, N, K)
    x = _x(rng, M, K)
    bias = rng.standard_normal(N).astype(np.float32)
    res = rng.standard_normal((M, N)).astype(np.float32)
    y = G.mul_mat(wtype, wq, wd, N, K, G.dev(x), M, bias=G.dev(bias), residual=G.dev(res), tc=True)
    assert G.lib().gb_gemm_tc_error() == 0
    ref = res + (O.mul_mat(wtype, w, N, K, x) + bias[None, :]).astype(np.float32)
    assert np.max(np.abs(y - ref)) <= 1e-5 * np.max(np.abs(ref))


@pytest.mark.parametrize("wtype", [O.Q8_0, O.Q4_0])
@pytest.mark.parametrize("N,K", [(4096, 4096), (14336, 4096), (4096, 14336), (128256, 4096),
                                 (10240, 14336)])
def test_operator_sweep_shapes_sampled_rows(G, wtype, N, K):
    """Operator-sweep shapes at full size; the oracle checks a sample of output rows (decode M=1,
    batched decode M=8 and 16, prefill M=64, within 1e-5 of the output range).  K = 14336 runs
    the batched decode kernel in several activation phases; 10240 rows give its CTAs more than
    one chunk of tiles."""
    torch = G.torch_dev()
    rng = np.random.default_rng(N ^ K ^ wtype)
    w = G.random_blocks(rng, wtype, N, K, scale=0.02 / 127 * 3)
    wq, wd = G.upload_weight(wtype, w, N, K)
    rows = np.sort(rng.choice(N, size=48, replace=False))
    for M in (1, 8, 16, 64):
        x = rng.standard_normal((M, K)).astype(np.float32)
        y = G.mul_mat(wtype, wq, wd, N, K, G.dev(x), M)
        ref = O.mul_mat(wtype, np.ascontiguousarray(w[rows]), len(rows), K, x)
        assert _close(y[:, rows], ref)
    del wq, wd
    torch.cuda.empty_cache()


@pytest.mark.parametrize("wtype", [O.Q8_0, O.Q4_0])
def test_get_rows_bit_exact(G, wtype):
    torch = G.torch_dev()
    rng = np.random.default_rng(3)
    V, K = 500, 256
    w = G.random_blocks(rng, wtype, V, K)
    wq, wd = G.upload_weight(wtype, w, V, K)
    ids = rng.integers(0, V, 37).astype(np.int32)
    ids_d = G.dev(ids)
    out = torch.empty((37, K), dtype=torch.float32, device="cuda")
    G.check(G.lib().gb_get_rows(wtype, G.ptr(wq), V, K, G.ptr(ids_d), 37,
                                G.ptr(out), None))
    ref = np.empty((37, K), np.float32)
    O.lib().oracle_get_rows(wtype, O._p(np.ascontiguousarray(w)), K, O._p(ids), 37, O._p(ref))
    assert np.array_equal(out.cpu().numpy(), ref)


@pytest.mark.parametrize("D", [256, 576, 4096])
def test_rms_norm_bit_exact(G, D):
    torch = G.torch_dev()
    rng = np.random.default_rng(D)
    M = 5
    x = (rng.standard_normal((M, D)) * 3).astype(np.float32)
    gam = rng.standard_normal(D).astype(np.float32)
    for gamma in (None, gam):
        y = torch.empty((M, D), dtype=torch.float32, device="cuda")
        yq = torch.empty((M, D), dtype=torch.int8, device="cuda")
        yd = torch.empty((M, D // 32), dtype=torch.float32, device="cuda")
        gd = None if gamma is None else G.dev(gamma)
        xd_ = G.dev(x)
        G.check(G.lib().gb_rms_norm(G.ptr(xd_), M, D, 1e-5, G.ptr(gd), G.ptr(y), G.ptr(yq),
                                    G.ptr(yd), None))
        ref = O.rms_norm(x, 1e-5, gamma)
        assert np.array_equal(y.cpu().numpy(), ref)
        refq = O.quantize_q8_0(ref).reshape(M, D // 32, 34)
        assert np.array_equal(yq.cpu().numpy(), refq[:, :, 2:].reshape(M, D).view(np.int8))


def _q8_agree(yq, ref_f32):
    """Q8_0 quants of the engine against the oracle's quantization of its f32 reference: the
    fraction of equal quants, and the largest difference"""
    M, D = ref_f32.shape
    refq = O.quantize_q8_0(ref_f32).reshape(M, D // 32, 34)[:, :, 2:].reshape(M, D).view(np.int8)
    d = np.abs(yq.astype(np.int32) - refq.astype(np.int32))
    return float((d == 0).mean()), int(d.max())


@pytest.mark.parametrize("D", [768, 4096])
def test_layer_norm_matches_oracle(G, D):
    """LayerNorm of the GPT-2 blocks (the CPU NORM op, ggml-cpu/ops.cpp:3762, restated in the
    oracle and pinned through the GPT-2 fixture's model-level goldens) with and without gamma /
    beta, f32 rows and the fused Q8_0 rows: fp32 rows within 2 ulp-sized relative error (the
    mean and variance are summed in double in another order), quants equal but for rare
    one-step flips at rounding ties (against the oracle and against the engine's own rows)."""
    torch = G.torch_dev()
    rng = np.random.default_rng(D + 1)
    M = 5
    x = (rng.standard_normal((M, D)) * 3 + 0.5).astype(np.float32)
    gam = rng.standard_normal(D).astype(np.float32)
    bet = rng.standard_normal(D).astype(np.float32)
    for gamma, beta in ((None, None), (gam, bet)):
        y = torch.empty((M, D), dtype=torch.float32, device="cuda")
        yq = torch.empty((M, D), dtype=torch.int8, device="cuda")
        yd = torch.empty((M, D // 32), dtype=torch.float32, device="cuda")
        gd = None if gamma is None else G.dev(gamma)
        bd = None if beta is None else G.dev(beta)
        xd_ = G.dev(x)
        G.check(G.lib().gb_layer_norm(G.ptr(xd_), M, D, 1e-5, G.ptr(gd), G.ptr(bd), G.ptr(y),
                                      G.ptr(yq), G.ptr(yd), None))
        ref = O.layer_norm(x, 1e-5, gamma, beta)
        out = y.cpu().numpy()
        np.testing.assert_allclose(out, ref, rtol=2.5e-7 * 2, atol=1e-6)
        same, worst = _q8_agree(yq.cpu().numpy(), out)
        assert same >= 0.999 and worst <= 1, ("fused Q8_0 against its own f32 rows", same, worst)
        same, worst = _q8_agree(yq.cpu().numpy(), ref)
        assert same >= 0.999 and worst <= 1, (same, worst)


@pytest.mark.parametrize("F", [128, 3072])
def test_bias_gelu_matches_oracle(G, F):
    """bias + tanh-GELU of the GPT-2 MLP (ggmlc's CPU custom op, stdlib_kernels.cpp:29, restated
    in the oracle and pinned through the GPT-2 fixture's goldens): f32 rows within 1e-6
    relative / 5e-7 absolute error, the fused Q8_0 rows those rows' quantization but for rare
    one-step flips."""
    torch = G.torch_dev()
    rng = np.random.default_rng(F + 3)
    M = 4
    x = (rng.standard_normal((M, F)) * 3).astype(np.float32)
    b = rng.standard_normal(F).astype(np.float32)
    y = torch.empty((M, F), dtype=torch.float32, device="cuda")
    yq = torch.empty((M, F), dtype=torch.int8, device="cuda")
    yd = torch.empty((M, F // 32), dtype=torch.float32, device="cuda")
    xd_, bd_ = G.dev(x), G.dev(b)  # held: a freed temporary's memory could be reused
    G.check(G.lib().gb_bias_gelu(G.ptr(xd_), G.ptr(bd_), M, F, G.ptr(y), G.ptr(yq), G.ptr(yd),
                                 None))
    ref = O.bias_gelu(x, b)
    out = y.cpu().numpy()
    # the CPU's libm expf is off by one ulp in rare cases and 1 + tanh cancels near the
    # negative tail, so a few near-zero outputs differ by about 1e-7 absolute
    np.testing.assert_allclose(out, ref, rtol=1e-6, atol=5e-7)
    same, worst = _q8_agree(yq.cpu().numpy(), out)
    assert same >= 0.999 and worst <= 1, ("fused Q8_0 against its own f32 rows", same, worst)


@pytest.mark.parametrize("F", [96, 1536, 14336])
def test_swiglu_bit_exact(G, F):
    torch = G.torch_dev()
    rng = np.random.default_rng(F)
    M = 3
    x = (rng.standard_normal((M, 2 * F)) * 4).astype(np.float32)
    x[0, :8] = [-120.0, -90.0, 88.0, 100.0, -1e-8, 0.0, 30.0, -30.0]  # exp special paths
    y = torch.empty((M, F), dtype=torch.float32, device="cuda")
    x_d = G.dev(x)
    G.check(G.lib().gb_swiglu(G.ptr(x_d), M, F, G.ptr(y), None, None, None))
    assert np.array_equal(y.cpu().numpy(), O.swiglu(x))


@pytest.mark.parametrize("base", [10000.0009765625, 500000.0])
def test_rope_bit_exact(G, base):
    torch = G.torch_dev()
    rng = np.random.default_rng(11)
    s, H, hd = 9, 4, 128
    x = rng.standard_normal((s, H, hd)).astype(np.float32)
    pos = np.array([0, 1, 2, 63, 64, 511, 900, 2047, 3000], np.int32)
    n_pos = 4096
    tab = np.empty((n_pos, hd // 2, 2), np.float32)
    G.lib().gb_rope_table_fill(tab.ctypes.data, n_pos, hd, base)
    y = torch.empty((s, H, hd), dtype=torch.float32, device="cuda")
    x_d, pos_d, tab_d = G.dev(x), G.dev(pos), G.dev(tab)  # keep device buffers alive
    G.check(G.lib().gb_rope_neox(G.ptr(x_d), hd, H, s, G.ptr(pos_d), hd, base, G.ptr(tab_d),
                                 n_pos, G.ptr(y), None))
    ref = O.rope_neox(x, pos, hd, np.float32(base))
    assert np.array_equal(y.cpu().numpy(), ref)


def _attention_exact(q, k, v, kv_pos, scale):
    """float64 attention with the CPU's fp16 rounding of Q (q_to_vec_dot) and causal rows."""
    s, Hq, hd = q.shape
    Hkv = k.shape[0]
    qh = q.astype(np.float16).astype(np.float64)
    out = np.zeros((s, Hq, hd))
    for t in range(s):
        n = kv_pos + t + 1
        for h in range(Hq):
            kk = k[h // (Hq // Hkv), :n].astype(np.float64)
            vv = v[h // (Hq // Hkv), :n].astype(np.float64)
            sc = kk @ qh[t, h] * scale
            p = np.exp(sc - sc.max())
            out[t, h] = p @ vv / p.sum()
    return out


@pytest.mark.parametrize("s,kv_pos,Hq,Hkv,hd", [(1, 40, 4, 2, 64), (1, 700, 32, 8, 128),
                                                (5, 100, 9, 3, 64), (70, 0, 4, 4, 64),
                                                (128, 300, 32, 8, 128), (33, 17, 9, 3, 64),
                                                (16, 0, 12, 12, 64)])
def test_attention_close(G, s, kv_pos, Hq, Hkv, hd):
    """Attention against an exact float64 evaluation: never further from it than the CPU's
    fp16-accumulator kernel (the oracle) is, and within 1e-5 of the output range for the
    fp32-accumulating CUDA-core kernel (s < 16) or 1e-3 for the tensor-core kernel (s >= 16,
    whose probabilities enter the second product as fp16)."""
    torch = G.torch_dev()
    rng = np.random.default_rng(s + kv_pos)
    ctx = 1024
    q = rng.standard_normal((s, Hq, hd)).astype(np.float32)
    k = rng.standard_normal((Hkv, ctx, hd)).astype(np.float16)
    v = rng.standard_normal((Hkv, ctx, hd)).astype(np.float16)
    scale = float(np.float32(1.0) / np.sqrt(np.float32(hd)))
    wb = G.lib().gb_attention_workspace_bytes(s, Hq, hd, ctx)
    work = torch.empty(max(int(wb), 16), dtype=torch.uint8, device="cuda")
    o = torch.empty((s, Hq, hd), dtype=torch.float32, device="cuda")
    q_d, k_d, v_d = G.dev(q), G.dev(k.view(np.uint16)), G.dev(v.view(np.uint16))
    G.check(G.lib().gb_attention(G.ptr(q_d), G.ptr(k_d), G.ptr(v_d), hd, s, Hq, Hkv, ctx, kv_pos,
                                 scale, G.ptr(o), G.ptr(work), None))
    got = o.cpu().numpy()
    exact = _attention_exact(q, k, v, kv_pos, scale)
    n_kv = kv_pos + s
    mask = O.causal_mask_f16(kv_pos, s, n_kv)
    cpu = O.flash_attn(q, np.ascontiguousarray(k[:, :n_kv]).view(np.uint16),
                       np.ascontiguousarray(v[:, :n_kv]).view(np.uint16), mask, np.float32(scale))
    err_gpu = np.max(np.abs(got - exact))
    err_cpu = np.max(np.abs(cpu - exact))
    assert err_gpu <= (1e-5 if s < 16 else 1e-3) * np.max(np.abs(exact))
    assert err_gpu <= err_cpu + 1e-6


@pytest.mark.parametrize("wtype", [O.Q8_0, O.Q4_0])
@pytest.mark.parametrize("M,K", [(1, 576), (1, 4096), (3, 1024)])
@pytest.mark.parametrize("with_gamma", [False, True])
def test_gemv_rms_prologue(G, wtype, M, K, with_gamma):
    """RMSNorm (+gamma) and Q8_0 quantization fused into the GEMV prologue: close to the
    tensor-core matmul fed by the standalone RMSNorm's Q8_0 output (itself bit-exact with the
    CPU) and to the oracle."""
    torch = G.torch_dev()
    rng = np.random.default_rng(K + M)
    N = 96
    w = G.random_blocks(rng, wtype, N, K)
    wq, wd = G.upload_weight(wtype, w, N, K)
    x = (rng.standard_normal((M, K)) * 2).astype(np.float32)
    gamma = rng.standard_normal(K).astype(np.float32) if with_gamma else None
    x_d = G.dev(x)
    g_d = G.dev(gamma) if with_gamma else None
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    L = G.lib_fused()
    G.check(L.gb_gemv(wtype, G.ptr(wq), N, K, M, None, None, G.ptr(x_d), 1e-5, G.ptr(g_d), 0,
                      G.ptr(y), None, None, None, None, None))
    xq = torch.empty((M, K), dtype=torch.int8, device="cuda")
    xd = torch.empty((M, K // 32), dtype=torch.float32, device="cuda")
    G.check(G.lib().gb_rms_norm(G.ptr(x_d), M, K, 1e-5, G.ptr(g_d), None, G.ptr(xq), G.ptr(xd),
                                None))
    y2 = torch.empty((M, N), dtype=torch.float32, device="cuda")
    G.check(L.gb_gemv(wtype, G.ptr(wq), N, K, M, G.ptr(xq), G.ptr(xd), None, 0.0, None, 0,
                      G.ptr(y2), None, None, None, None, None))
    ref = O.mul_mat(wtype, w, N, K, O.rms_norm(x, 1e-5, gamma))
    assert _close(y.cpu().numpy(), ref)
    assert _close(y2.cpu().numpy(), ref)
    assert _close(y.cpu().numpy(), y2.cpu().numpy())


@pytest.mark.parametrize("wtype", [O.Q8_0, O.Q4_0])
@pytest.mark.parametrize("M", [1, 2, 7, 16])
def test_gemv_swiglu_epilogue(G, wtype, M):
    """gate_up matmul with SwiGLU and Q8_0 quantization of the result fused in the epilogue:
    bit-exact with the CPU SwiGLU and quantizer applied to the plain matmul's outputs (both
    modes build every output from the same partial sums)."""
    torch = G.torch_dev()
    rng = np.random.default_rng(M)
    F, K = 160, 512
    N = 2 * F
    w = G.random_blocks(rng, wtype, N, K, scale=0.05)
    wq, wd = G.upload_weight(wtype, w, N, K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    xq, xd = G.quantize(G.dev(x), M, K)
    y = torch.empty((M, F), dtype=torch.float32, device="cuda")
    yq = torch.empty((M, F), dtype=torch.int8, device="cuda")
    yd = torch.empty((M, F // 32), dtype=torch.float32, device="cuda")
    L = G.lib_fused()
    G.check(L.gb_gemv(wtype, G.ptr(wq), N, K, M, G.ptr(xq), G.ptr(xd), None, 0.0, None, 1,
                      G.ptr(y), G.ptr(yq), G.ptr(yd), None, None, None))
    gu = torch.empty((M, N), dtype=torch.float32, device="cuda")
    G.check(L.gb_gemv(wtype, G.ptr(wq), N, K, M, G.ptr(xq), G.ptr(xd), None, 0.0, None, 0,
                      G.ptr(gu), None, None, None, None, None))
    h = O.swiglu(gu.cpu().numpy())
    assert np.array_equal(y.cpu().numpy(), h)
    hq = O.quantize_q8_0(h).reshape(M, F // 32, 34)
    assert np.array_equal(yq.cpu().numpy(), hq[:, :, 2:].reshape(M, F).view(np.int8))
    assert np.array_equal(yd.cpu().numpy(),
                          hq[:, :, :2].copy().view(np.float16).reshape(M, F // 32).astype(np.float32))
    assert _close(h, O.swiglu(O.mul_mat(wtype, w, N, K, x)), 1e-4)


@pytest.mark.parametrize("Hq,Hkv,hd,kv_pos,ctx", [(4, 2, 64, 0, 1024), (9, 3, 64, 300, 1024),
                                                  (32, 8, 128, 700, 1024), (9, 3, 64, 1200, 2048),
                                                  (32, 8, 128, 1500, 2048),
                                                  (32, 8, 128, 6000, 8192)])
def test_attn_decode_fused(G, Hq, Hkv, hd, kv_pos, ctx):
    """Decode attention fused with RoPE and the KV write: cache row kv_pos holds fp16(rope(k)) and
    fp16(v) bit-exactly, the output matches exact fp64 attention over the rotated q.  Caches of
    1024-2048 positions run as one launch whose thread-block clusters merge their CTAs' partials
    in distributed shared memory; the 8192-position cache takes the wider split and the merge
    launch."""
    torch = G.torch_dev()
    rng = np.random.default_rng(Hq + kv_pos)
    base = 500000.0
    qkv = rng.standard_normal((Hq + 2 * Hkv) * hd).astype(np.float32)
    k = rng.standard_normal((Hkv, ctx, hd)).astype(np.float16)
    v = rng.standard_normal((Hkv, ctx, hd)).astype(np.float16)
    n_pos = max(4096, ctx)
    tab = np.empty((n_pos, hd // 2, 2), np.float32)
    L = G.lib_fused()
    G.lib().gb_rope_table_fill(tab.ctypes.data, n_pos, hd, base)
    scale = float(np.float32(1.0) / np.sqrt(np.float32(hd)))
    wb = L.gb_attn_decode_workspace_bytes(Hq, Hkv, hd, ctx)
    work = torch.empty(int(wb), dtype=torch.uint8, device="cuda")
    q_d, k_d, v_d, t_d = G.dev(qkv), G.dev(k.view(np.uint16)), G.dev(v.view(np.uint16)), G.dev(tab)
    o = torch.empty((Hq, hd), dtype=torch.float32, device="cuda")
    oq = torch.empty(Hq * hd, dtype=torch.int8, device="cuda")
    od = torch.empty(Hq * hd // 32, dtype=torch.float32, device="cuda")
    G.check(L.gb_attn_decode(G.ptr(q_d), Hq, Hkv, hd, G.ptr(k_d), G.ptr(v_d), ctx, kv_pos, hd,
                             base, G.ptr(t_d), n_pos, scale, G.ptr(o), G.ptr(oq), G.ptr(od),
                             G.ptr(work), None))
    pos = np.array([kv_pos], np.int32)
    qr = O.rope_neox(qkv[: Hq * hd].reshape(1, Hq, hd), pos, hd, np.float32(base))[0]
    kr = O.rope_neox(qkv[Hq * hd:(Hq + Hkv) * hd].reshape(1, Hkv, hd), pos, hd, np.float32(base))[0]
    vn = qkv[(Hq + Hkv) * hd:].reshape(Hkv, hd)
    kc = k_d.cpu().numpy().view(np.float16)
    vc = v_d.cpu().numpy().view(np.float16)
    assert np.array_equal(kc[:, kv_pos], kr.astype(np.float16))
    assert np.array_equal(vc[:, kv_pos], vn.astype(np.float16))
    k2 = k.copy()
    v2 = v.copy()
    k2[:, kv_pos] = kr.astype(np.float16)
    v2[:, kv_pos] = vn.astype(np.float16)
    exact = _attention_exact(qr.reshape(1, Hq, hd), k2, v2, kv_pos, scale)[0]
    got = o.cpu().numpy()
    assert np.max(np.abs(got - exact)) <= 1e-5 * np.max(np.abs(exact))
    ref_q = O.quantize_q8_0(got.reshape(1, -1)).reshape(-1, 34)
    assert np.array_equal(oq.cpu().numpy(), ref_q[:, 2:].reshape(-1).view(np.int8))


@pytest.mark.parametrize("wtype", [O.Q8_0, O.Q4_0])
@pytest.mark.parametrize("K", [576, 4096, 14336])
@pytest.mark.parametrize("M", [1, 2])
def test_gemv_bulk_copy_rows(G, wtype, K, M):
    """The 1-2-row decode GEMV (weight rows streamed by bulk copies into per-warp rings; K up to
    4096 keeps the activations in registers, longer rows read them from shared memory):
    bit-exact with the oracle where fp32 summation is exact, with bias and residual; its SwiGLU
    mode equals the CPU SwiGLU of its own plain outputs; its RMSNorm prologue gives the same
    bits as the standalone RMSNorm's Q8_0 rows fed to it; its error word stays clear."""
    torch = G.torch_dev()
    rng = np.random.default_rng(K * 3 + M + wtype)
    F = 72
    N = 2 * F
    w, x = _int_exact_case(rng, wtype, N, K, M)
    wq, wd = G.upload_weight(wtype, w, N, K)
    bias = rng.integers(-4, 5, size=N).astype(np.float32)
    res = rng.integers(-4, 5, size=(M, N)).astype(np.float32)
    L = G.lib_fused()
    xq, xd = G.quantize(G.dev(x), M, K)
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    bias_d, res_d = G.dev(bias), G.dev(res)  # held: the launch reads them asynchronously
    G.check(L.gb_gemv(wtype, G.ptr(wq), N, K, M, G.ptr(xq), G.ptr(xd), None, 0.0, None, 0,
                      G.ptr(y), None, None, G.ptr(bias_d), G.ptr(res_d), None))
    ref = res + (O.mul_mat(wtype, w, N, K, x) + bias[None, :]).astype(np.float32)
    assert np.array_equal(y.cpu().numpy(), ref.astype(np.float32))
    # SwiGLU of row pairs (n, n + F), f32 out
    wr = G.random_blocks(rng, wtype, N, K, scale=0.05)
    wq2, _ = G.upload_weight(wtype, wr, N, K)
    xr = rng.standard_normal((M, K)).astype(np.float32)
    xq2, xd2 = G.quantize(G.dev(xr), M, K)
    gu = torch.empty((M, N), dtype=torch.float32, device="cuda")
    G.check(L.gb_gemv(wtype, G.ptr(wq2), N, K, M, G.ptr(xq2), G.ptr(xd2), None, 0.0, None, 0,
                      G.ptr(gu), None, None, None, None, None))
    h = torch.empty((M, F), dtype=torch.float32, device="cuda")
    G.check(L.gb_gemv(wtype, G.ptr(wq2), N, K, M, G.ptr(xq2), G.ptr(xd2), None, 0.0, None, 1,
                      G.ptr(h), None, None, None, None, None))
    assert np.array_equal(h.cpu().numpy(), O.swiglu(gu.cpu().numpy()))
    assert _close(gu.cpu().numpy(), O.mul_mat(wtype, wr, N, K, xr))
    # RMSNorm + gamma prologue: the same bits as the standalone RMSNorm's Q8_0 rows
    gamma = rng.standard_normal(K).astype(np.float32)
    x_d, g_d = G.dev(xr * 3), G.dev(gamma)
    yf = torch.empty((M, N), dtype=torch.float32, device="cuda")
    G.check(L.gb_gemv(wtype, G.ptr(wq2), N, K, M, None, None, G.ptr(x_d), 1e-5, G.ptr(g_d), 0,
                      G.ptr(yf), None, None, None, None, None))
    nq = torch.empty((M, K), dtype=torch.int8, device="cuda")
    nd = torch.empty((M, K // 32), dtype=torch.float32, device="cuda")
    G.check(G.lib().gb_rms_norm(G.ptr(x_d), M, K, 1e-5, G.ptr(g_d), None, G.ptr(nq), G.ptr(nd),
                                None))
    yq_ = torch.empty((M, N), dtype=torch.float32, device="cuda")
    G.check(L.gb_gemv(wtype, G.ptr(wq2), N, K, M, G.ptr(nq), G.ptr(nd), None, 0.0, None, 0,
                      G.ptr(yq_), None, None, None, None, None))
    assert torch.equal(yf, yq_)
    L.gb_gemv_error.restype = ctypes.c_int
    assert L.gb_gemv_error() == 0
