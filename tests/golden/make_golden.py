"""Writes the golden fixtures under tests/golden/ from the reference itself.

Run in a container that has the reference checkout (default /root/reference, or $GGMLC_REF) and a
built oracle/_ref (``make -C oracle``):

    python tests/golden/make_golden.py               # everything
    python tests/golden/make_golden.py --batch-only  # the per-sequence batch goldens only
    python tests/golden/make_golden.py --kv8-only    # the eight-KV-head Llama only

1. Seeded random-init HF models (transformers, no network) wrapped with the reference's own
   wrappers (examples/models/hub_models.py: load_smollm2_model :366, load_gpt2_model :47) and
   compiled by the reference compiler ``ggmlc.compile`` (python/ggmlc/compiler.py:138) to GGUF.
2. Golden outputs from the reference CPU code (oracle/_ref/libggmlc_ref.so, built from the
   reference sources): op-level vectors through one-op ggml graphs and model-level logits and
   greedy tokens through ggmlc::ModelExecutor with the padded KV cache.

The GGUFs and .npz files are committed; this script is only needed to regenerate them.  The
committed files were written with NumPy 2.3.5: the compiler's RoPE freq_base recovery
(python/ggmlc/transforms/fusion.py:322, ``(1.0 / arr[1]) ** (n_dims / 2.0)`` on a float32 array
element) stays in float32 under NumPy 2's scalar promotion and would promote to float64 under
NumPy 1.x, which can move the recorded freq_base (and every RoPE angle after it).  The script
refuses to run under NumPy 1.x for that reason.
"""

from __future__ import annotations

import ctypes
import os
import sys
from pathlib import Path
from unittest import mock

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
REF = Path(os.environ.get("GGMLC_REF", "/root/reference"))
REF_LIB = REPO / "oracle" / "_ref" / "libggmlc_ref.so"


def ref_lib():
    L = ctypes.CDLL(str(REF_LIB))
    P, I64, F, I = ctypes.c_void_p, ctypes.c_int64, ctypes.c_float, ctypes.c_int
    L.ref_quantize_row_q8_0.argtypes = [P, P, I64]
    L.ref_dequantize_row.argtypes = [I, P, P, I64]
    L.ref_vec_dot.argtypes = [I, I, P, P, P]
    L.ref_mul_mat.argtypes = [I, P, I64, I64, P, I64, P, I]
    L.ref_rms_norm.argtypes = [P, I64, I64, F, P, P, I]
    L.ref_rope_neox.argtypes = [P, I64, I64, I64, P, I, F, P, I]
    L.ref_swiglu.argtypes = [P, I64, I64, P, I]
    L.ref_flash_attn.argtypes = [P, P, P, P, I64, I64, I64, I64, I64, F, P, I]
    L.ref_model_open.argtypes = [ctypes.c_char_p, I]
    L.ref_model_open.restype = P
    L.ref_model_close.argtypes = [P]
    L.ref_model_init_kv.argtypes = [P, I64]
    L.ref_model_reset_kv.argtypes = [P]
    L.ref_model_set_logits_last_only.argtypes = [P, I]
    L.ref_model_forward.argtypes = [P, P, I64, I64, P, I64]
    L.ref_model_forward.restype = I64
    L.ref_last_error.restype = ctypes.c_char_p
    return L


def p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


# Tiny model shapes (head_dim 64 keeps the reference on its FLASH_ATTN_EXT path,
# executor.cpp:2305-2308).
LLAMA = dict(L=2, d=256, hq=4, hkv=2, hd=64, ffn=512, V=512)
# eight KV heads, so tensor parallelism over 2, 4 and 8 ranks each keeps whole heads
LLAMA_KV8 = dict(L=2, d=512, hq=8, hkv=8, hd=64, ffn=1024, V=512)
GPT2 = dict(L=2, d=256, nh=4, ffn=1024, V=500, npos=512)


def compile_llama(out: Path, quant: str, theta: float, seed: int, shape: dict = LLAMA,
                  name: str = "tiny_llama"):
    sys.path.insert(0, str(REF / "python"))
    sys.path.insert(0, str(REF))
    import torch
    import transformers
    from transformers import LlamaConfig, LlamaForCausalLM

    import ggmlc
    from examples.models import hub_models

    torch.manual_seed(seed)
    c = shape
    cfg = LlamaConfig(hidden_size=c["d"], num_hidden_layers=c["L"], num_attention_heads=c["hq"],
                      num_key_value_heads=c["hkv"], head_dim=c["hd"], intermediate_size=c["ffn"],
                      vocab_size=c["V"], rms_norm_eps=1e-5, rope_theta=theta,
                      tie_word_embeddings=True, initializer_range=0.02)
    model = LlamaForCausalLM(cfg).eval()
    with mock.patch.object(transformers.AutoModelForCausalLM, "from_pretrained",
                           return_value=model):
        m, dummy, _ = hub_models.load_smollm2_model(seq_len=8)
    dim_s = torch.export.Dim("s", min=1, max=2048)
    ggmlc.compile(m, dummy, output=str(out), dynamic_shapes=({1: dim_s},), model_name=name,
                  quantize=quant, tasks=["text-generation"])


def compile_gpt2(out: Path, seed: int):
    sys.path.insert(0, str(REF / "python"))
    sys.path.insert(0, str(REF))
    import torch
    import transformers
    from transformers import GPT2Config, GPT2LMHeadModel

    import ggmlc
    from examples.models import hub_models

    torch.manual_seed(seed)
    c = GPT2
    cfg = GPT2Config(n_embd=c["d"], n_layer=c["L"], n_head=c["nh"], n_inner=c["ffn"],
                     n_positions=c["npos"], vocab_size=c["V"], tie_word_embeddings=True,
                     initializer_range=0.02)
    model = GPT2LMHeadModel(cfg).eval()
    with mock.patch.object(transformers.GPT2LMHeadModel, "from_pretrained", return_value=model):
        m, dummy, _ = hub_models.load_gpt2_model(seq_len=8)
    dim_s = torch.export.Dim("s", min=1, max=c["npos"])
    ggmlc.compile(m, dummy, output=str(out), dynamic_shapes=({1: dim_s}, {1: dim_s}),
                  model_name="tiny_gpt2", quantize="q8_0", tasks=["text-generation"])


def model_golden(L, gguf: Path, V: int, prompt_len: int, n_decode: int, seed: int,
                 max_ctx: int = 1024):
    """Prefill logits (full sequence, no KV) + greedy decode through the padded KV cache."""
    rng = np.random.default_rng(seed)
    prompt = rng.integers(0, V, size=prompt_len, dtype=np.int32)
    h = L.ref_model_open(str(gguf).encode(), 1)
    assert h, L.ref_last_error()
    out = np.empty(V * max_ctx, np.float32)
    # plain forward over the prompt (no KV cache)
    n = L.ref_model_forward(h, p(prompt), prompt_len, -1, p(out), out.size)
    assert n > 0, L.ref_last_error()
    full_logits = out[:n].reshape(prompt_len, V).copy()
    L.ref_model_close(h)
    # KV path: prefill then greedy decode, one token per step
    h = L.ref_model_open(str(gguf).encode(), 1)
    assert L.ref_model_init_kv(h, max_ctx) == 1, L.ref_last_error()
    n = L.ref_model_forward(h, p(prompt), prompt_len, 0, p(out), out.size)
    assert n > 0, L.ref_last_error()
    kv_prefill = out[:n].reshape(prompt_len, V).copy()
    tokens = [int(np.argmax(kv_prefill[-1]))]
    dec_logits = []
    pos = prompt_len
    for _ in range(n_decode):
        t = np.array([tokens[-1]], np.int32)
        n = L.ref_model_forward(h, p(t), 1, pos, p(out), out.size)
        assert n == V, L.ref_last_error()
        dec_logits.append(out[:V].copy())
        tokens.append(int(np.argmax(out[:V])))
        pos += 1
    L.ref_model_close(h)
    return dict(prompt=prompt, full_logits=full_logits, kv_prefill_logits=kv_prefill,
                decode_logits=np.stack(dec_logits), greedy_tokens=np.array(tokens, np.int32))


def batch_golden(L, gguf: Path, V: int, lengths: list[int], n_decode: int, seed: int,
                 max_ctx: int = 1024):
    """Several independent sequences through the reference's KV path, one executor each: for
    prompt k (lengths[k] tokens), its greedy tokens and the logits row each token was chosen
    from (row 0: the prefill's last row; row i: after feeding token i - 1 at position
    lengths[k] + i - 1).  The oracle of batched decode: every row of a batched step must follow
    its own sequence's reference run."""
    rng = np.random.default_rng(seed)
    prompts, toks, rows = [], [], []
    out = np.empty(V * max_ctx, np.float32)
    for n_p in lengths:
        prompt = rng.integers(1, V, size=n_p, dtype=np.int32)
        h = L.ref_model_open(str(gguf).encode(), 1)
        assert h and L.ref_model_init_kv(h, max_ctx) == 1, L.ref_last_error()
        n = L.ref_model_forward(h, p(prompt), n_p, 0, p(out), out.size)
        assert n > 0, L.ref_last_error()
        r = [out[(n_p - 1) * V:n_p * V].copy()]
        t = [int(np.argmax(r[0]))]
        for i in range(n_decode):
            x = np.array([t[-1]], np.int32)
            n = L.ref_model_forward(h, p(x), 1, n_p + i, p(out), out.size)
            assert n == V, L.ref_last_error()
            r.append(out[:V].copy())
            t.append(int(np.argmax(out[:V])))
        L.ref_model_close(h)
        prompts.append(prompt)
        toks.append(t)
        rows.append(np.stack(r))
    return dict(lengths=np.array(lengths, np.int32), prompts=np.concatenate(prompts),
                tokens=np.array(toks, np.int32), logits=np.stack(rows))


def op_golden(L, seed=7):
    rng = np.random.default_rng(seed)
    g = {}
    # activation quantization incl. exact .5 ties of x*id (x = (k+0.5)*amax/127)
    K = 256
    x = rng.standard_normal((4, K)).astype(np.float32)
    tie = np.zeros(K, np.float32)
    tie[0] = 127.0
    tie[1:64] = np.arange(63, dtype=np.float32) + 0.5
    tie[64:128] = -(np.arange(64, dtype=np.float32) + 0.5)
    x = np.concatenate([x, tie[None], np.zeros((1, K), np.float32)], 0)
    q = np.empty((x.shape[0], K // 32 * 34), np.uint8)
    L.ref_quantize_row_q8_0(p(x), p(q), x.size)
    g["quant_x"], g["quant_q8_0"] = x, q
    # weight blocks and int dots, per type
    for name, t, bb in (("q8_0", 8, 34), ("q4_0", 2, 18)):
        N = 64
        w = rng.integers(0, 256, size=(N, K // 32 * bb), dtype=np.uint8)
        if t == 8:  # Q8_0 quants are in [-127, 127]; -128 never occurs in valid blocks
            w[w == 128] = 129
        d = (rng.standard_normal((N, K // 32)) * 0.01).astype(np.float16)
        wv = w.reshape(N, K // 32, bb)
        wv[:, :, 0:2] = d.view(np.uint8).reshape(N, K // 32, 2)
        w = wv.reshape(N, -1)
        deq = np.empty((N, K), np.float32)
        L.ref_dequantize_row(t, p(w), p(deq), N * K)
        dots = np.empty((N, x.shape[0]), np.float32)
        for n in range(N):
            for m in range(x.shape[0]):
                s = np.zeros(1, np.float32)
                L.ref_vec_dot(t, K, p(s), p(w[n]), p(q[m]))
                dots[n, m] = s[0]
        g[f"w_{name}"], g[f"deq_{name}"], g[f"dot_{name}"] = w, deq, dots
        # MUL_MAT through the ggml graph (quantize + llamafile/vec_dot dispatch)
        M = 5
        xm = rng.standard_normal((M, K)).astype(np.float32)
        y = np.empty((M, N), np.float32)
        assert L.ref_mul_mat(t, p(w), N, K, p(xm), M, p(y), 1) == 0
        g[f"mm_x_{name}"], g[f"mm_y_{name}"] = xm, y
    # rms norm with and without gamma
    xr = (rng.standard_normal((3, 256)) * 2).astype(np.float32)
    gam = rng.standard_normal(256).astype(np.float32)
    y0 = np.empty_like(xr)
    y1 = np.empty_like(xr)
    L.ref_rms_norm(p(xr), 256, 3, 1e-5, None, p(y0), 1)
    L.ref_rms_norm(p(xr), 256, 3, 1e-5, p(gam), p(y1), 1)
    g["rms_x"], g["rms_gamma"], g["rms_y"], g["rms_y_gamma"] = xr, gam, y0, y1
    # NEOX rope at large positions (theta recurrence), two bases
    s, H, hd = 5, 3, 64
    xr = rng.standard_normal((s, H, hd)).astype(np.float32)
    pos = np.array([0, 1, 17, 900, 2047], np.int32)
    for tag, base in (("1e4", 10000.0009765625), ("5e5", 500000.0)):
        y = np.empty_like(xr)
        L.ref_rope_neox(p(xr), hd, H, s, p(pos), hd, base, p(y), 1)
        g[f"rope_y_{tag}"] = y
    g["rope_x"], g["rope_pos"] = xr, pos
    # swiglu
    xs = (rng.standard_normal((3, 2 * 96)) * 3).astype(np.float32)
    ys = np.empty((3, 96), np.float32)
    L.ref_swiglu(p(xs), 96, 3, p(ys), 1)
    g["swiglu_x"], g["swiglu_y"] = xs, ys
    # flash attention over an f16 cache with the executor's padded causal mask
    hd, s, Hq, Hkv, n_kv, pos0 = 64, 3, 4, 2, 256, 40
    qa = rng.standard_normal((s, Hq, hd)).astype(np.float32)
    ka = (rng.standard_normal((Hkv, n_kv, hd))).astype(np.float16)
    va = (rng.standard_normal((Hkv, n_kv, hd))).astype(np.float16)
    j = np.arange(n_kv)[None, :]
    i = np.arange(s)[:, None]
    mask = np.where(j <= pos0 + i, 0.0, -32768.0).astype(np.float16)
    qg = np.ascontiguousarray(np.transpose(qa, (1, 0, 2)))  # ggml ne [hd, s, Hq]
    y = np.empty((s, Hq, hd), np.float32)
    assert L.ref_flash_attn(p(qg), p(ka.view(np.uint16)), p(va.view(np.uint16)),
                            p(mask.view(np.uint16)), hd, s, Hq, Hkv, n_kv,
                            1.0 / np.sqrt(np.float32(hd)), p(y), 1) == 0
    g["fa_q"], g["fa_k"], g["fa_v"], g["fa_mask"], g["fa_y"] = qa, ka, va, mask, y
    g["fa_pos0"] = np.array([pos0])
    return g


def main_batch():
    """Only the per-sequence batch goldens, from the committed GGUFs (no recompilation)."""
    L = ref_lib()
    for fname in ("tiny_llama_q8_0.gguf", "tiny_llama_q4_0.gguf"):
        f = HERE / fname
        V = int(np.load(HERE / fname.replace(".gguf", ".npz"))["full_logits"].shape[1])
        gold = batch_golden(L, f, V, [5, 17, 33, 9, 40, 3], n_decode=10, seed=31)
        np.savez_compressed(HERE / fname.replace(".gguf", "_batch.npz"), **gold)
        print(fname, "batch tokens", gold["tokens"][:, :6].tolist())


def main_kv8():
    """Only the eight-KV-head Llama fixture (tensor parallelism over up to 8 ranks)."""
    L = ref_lib()
    f = HERE / "tiny_llama_kv8_q4_0.gguf"
    compile_llama(f, "q4_0", 500000.0, 3, LLAMA_KV8, "tiny_llama_kv8")
    gold = model_golden(L, f, LLAMA_KV8["V"], prompt_len=37, n_decode=12, seed=13)
    np.savez_compressed(HERE / "tiny_llama_kv8_q4_0.npz", **gold)
    print(f.name, f.stat().st_size, "tokens", gold["greedy_tokens"][:8])


def main():
    L = ref_lib()
    np.savez_compressed(HERE / "ops_golden.npz", **op_golden(L))
    fixtures = [
        ("tiny_llama_q8_0.gguf", lambda f: compile_llama(f, "q8_0", 10000.0, 0), LLAMA["V"]),
        ("tiny_llama_q4_0.gguf", lambda f: compile_llama(f, "q4_0", 500000.0, 1), LLAMA["V"]),
        ("tiny_gpt2_q8_0.gguf", lambda f: compile_gpt2(f, 2), GPT2["V"]),
    ]
    for fname, make, V in fixtures:
        f = HERE / fname
        make(f)
        gold = model_golden(L, f, V, prompt_len=37, n_decode=12, seed=11)
        np.savez_compressed(HERE / fname.replace(".gguf", ".npz"), **gold)
        print(fname, f.stat().st_size, "tokens", gold["greedy_tokens"][:8])
    main_batch()


if __name__ == "__main__":
    if int(np.__version__.split(".")[0]) < 2:
        sys.exit(f"NumPy {np.__version__}: the committed goldens follow NumPy 2 scalar promotion")
    if "--batch-only" in sys.argv:
        main_batch()
    elif "--kv8-only" in sys.argv:
        main_kv8()
    else:
        main()
        main_kv8()
