"""Kernel-level checks of the tcgen05 GEMM and the varlen attention against
a plain PyTorch fp32 reference of the same op (bf16 inputs)."""
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _gemm(ec, A, W, bias, resid, epi, bn, out_cols, out_dtype):
    M, K = A.shape
    N = W.shape[0]
    out = torch.empty((M, out_cols), dtype=out_dtype, device="cuda")
    torch.cuda.synchronize()
    ec.check(ec.lib().ecdbg_gemm(A.data_ptr(), W.data_ptr(), M, N, K,
                                 bias.data_ptr() if bias is not None else None,
                                 resid.data_ptr() if resid is not None else None,
                                 out.data_ptr(), epi, bn), "gemm")
    return out


def _gelu_as(x):
    # bert::gelu with the A&S erf (bert.lisp:176-192); |erf err| < 1.5e-7
    return 0.5 * x * (1.0 + torch.erf(x / math.sqrt(2.0)))


@pytest.mark.parametrize("M,N,K,bn", [
    (1, 384, 384, 0), (127, 1152, 384, 192), (128, 1152, 384, 128), (300, 1536, 384, 256),
    (4101, 384, 1536, 192), (777, 2304, 768, 256), (2048, 768, 3072, 0), (513, 1024, 2048, 128),
    (64, 256, 64, 64),
])
@pytest.mark.parametrize("epi", [0, 1, 2, 4])
def test_gemm_epilogues(ec, M, N, K, bn, epi):
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N + K + epi)
    A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    W = (0.05 * torch.randn(N, K, device="cuda", generator=g)).bfloat16()
    bias = torch.randn(N, device="cuda", generator=g)
    ref = A.float() @ W.float().t() + bias
    if epi in (0, 1):
        out = _gemm(ec, A, W, bias, None, epi, bn, N, torch.bfloat16).float()
        if epi == 1:
            ref = _gelu_as(ref)
        tol = 1e-2
    else:
        resid = torch.randn(M, N, device="cuda", generator=g) if epi == 2 else None
        if resid is not None:
            ref = ref + resid
        out = _gemm(ec, A, W, bias, resid, epi, bn, N, torch.float32)
        tol = 1e-4
    err = (out - ref).abs().max().item() / max(ref.abs().max().item(), 1e-6)
    assert err < tol, f"rel err {err}"


def _gelu_tanh(x):
    # gemma::gelu-tanh (gemma.lisp:85-89)
    return 0.5 * x * (1.0 + torch.tanh(0.7978845608028654 * (x + 0.044715 * x ** 3)))


# EmbeddingGemma epilogues: gelu_tanh(gate) * up on SwiGLU's 128-row
# interleave (6), and gelu_tanh(acc) * an fp32 multiplier (7, the PLE gate)
@pytest.mark.parametrize("M,N,K", [(1, 512, 512), (300, 4096, 512), (1029, 512, 512)])
@pytest.mark.parametrize("epi", [6, 7])
def test_gemm_gelu_tanh_epilogues(ec, M, N, K, epi):
    g = torch.Generator(device="cuda").manual_seed(M + N + epi)
    A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    if epi == 6:
        F = N // 2
        Wg = (0.05 * torch.randn(F, K, device="cuda", generator=g)).bfloat16()
        Wu = (0.05 * torch.randn(F, K, device="cuda", generator=g)).bfloat16()
        W = torch.stack([Wg.view(F // 128, 128, K), Wu.view(F // 128, 128, K)], 1).reshape(N, K)
        out = _gemm(ec, A, W.contiguous(), None, None, 6, 0, F, torch.bfloat16).float()
        ref = _gelu_tanh(A.float() @ Wg.float().t()) * (A.float() @ Wu.float().t())
    else:
        W = (0.05 * torch.randn(N, K, device="cuda", generator=g)).bfloat16()
        mul = torch.randn(M, N, device="cuda", generator=g)
        out = _gemm(ec, A, W, None, mul, 7, 0, N, torch.bfloat16).float()
        ref = _gelu_tanh(A.float() @ W.float().t()) * mul
    err = (out - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1e-2, err


def _rms(x, eps):
    return x / torch.sqrt((x * x).mean(-1, keepdim=True) + eps)


# GEMM + RMSNorm epilogues on clusters (the Qwen3 residual add + pre-norm,
# Gemma's post-norm residual adds with and without the layer scalar and the
# second norm, Gemma's per-layer-input norm); in-place residual for mode 2
@pytest.mark.parametrize("M,N,K", [(1, 512, 512), (300, 512, 2048), (1029, 1024, 512),
                                   (777, 768, 768)])
@pytest.mark.parametrize("mode,variant", [(1, 0), (2, 0), (2, 1), (3, 0)])
def test_gemm_rms_epilogues(ec, M, N, K, mode, variant):
    import ctypes as C
    g = torch.Generator(device="cuda").manual_seed(M + N + K + mode)
    A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    W = (0.05 * torch.randn(N, K, device="cuda", generator=g)).bfloat16()
    g1 = 1 + 0.1 * torch.randn(N, device="cuda", generator=g)
    g2 = 1 + 0.1 * torch.randn(N, device="cuda", generator=g)
    resid = torch.randn(M, N, device="cuda", generator=g)
    x = A.float() @ W.float().t()
    eps, scale = 1e-6, 0.75
    out32 = resid.clone() if mode == 2 else torch.empty(M, N, device="cuda")
    outb = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    if mode == 1:
        ref32 = x + resid
        refb = _rms(ref32, eps) * g1
        args = (resid.data_ptr(), g1.data_ptr(), None, 0, 1.0)
    elif mode == 2:
        ref32 = resid + _rms(x, eps) * g1
        if variant:
            ref32 = ref32 * scale
        refb = _rms(ref32, eps) * g2 if variant else ref32
        # in place: the residual is the fp32 output
        args = (out32.data_ptr(), g1.data_ptr(), g2.data_ptr() if variant else None, variant, scale)
    else:
        ref32 = _rms(x * scale, eps) * g1
        refb = ref32
        args = (None, g1.data_ptr(), None, 0, scale)
    resid_p, g1_p, g2_p, has_scale, sc = args
    torch.cuda.synchronize()
    ec.check(ec.lib().ecdbg_gemm_norm(A.data_ptr(), W.data_ptr(), M, N, K, resid_p, g1_p, g2_p,
                                      out32.data_ptr(), outb.data_ptr(), mode, eps, sc,
                                      has_scale), "gemm_norm")
    e32 = (out32 - ref32).abs().max().item() / ref32.abs().max().item()
    eb = (outb.float() - refb).abs().max().item() / refb.abs().max().item()
    assert e32 < 1e-4, e32
    assert eb < 1e-2, eb


# CTA-pair GEMM (cta_group::2, 256 x 256 tiles): ragged M (one or both
# halves of the last tile past M), K down to one k-block
@pytest.mark.parametrize("M,N,K", [(1, 256, 64), (129, 512, 384), (300, 1536, 384),
                                   (4097, 1536, 384), (2000, 768, 768), (513, 3072, 768)])
@pytest.mark.parametrize("epi", [0, 1, 2, 4])
def test_gemm_cta_pair(ec, monkeypatch, M, N, K, epi):
    monkeypatch.setenv("EC_GEMM_PAIR", "1")
    monkeypatch.setenv("EC_NO_GEMM_WR", "1")  # the streaming pair schedule, not weight-resident
    g = torch.Generator(device="cuda").manual_seed(M * 3 + N + K + epi)
    A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    W = (0.05 * torch.randn(N, K, device="cuda", generator=g)).bfloat16()
    bias = torch.randn(N, device="cuda", generator=g)
    ref = A.float() @ W.float().t() + bias
    if epi == 1:
        ref = _gelu_as(ref)
    if epi in (0, 1):
        out = _gemm(ec, A, W, bias, None, epi, 0, N, torch.bfloat16).float()
        tol = 1e-2
    else:
        resid = torch.randn(M, N, device="cuda", generator=g) if epi == 2 else None
        if resid is not None:
            ref = ref + resid
        out = _gemm(ec, A, W, bias, resid, epi, 0, N, torch.float32)
        tol = 1e-4
    err = (out - ref).abs().max().item() / max(ref.abs().max().item(), 1e-6)
    assert err < tol, f"rel err {err}"


# weight-resident CTA pairs (K <= 384, plain and GELU epilogues): each pair
# keeps one W tile in shared memory for the launch; units are grouped by W
# tile and share row blocks.  Ragged M (including fewer row blocks than
# groups), K of one k-block up to 384, W-tile counts from 1 to 16 (BN 192 and
# 256), and the equivalence with the streaming schedule.
@pytest.mark.parametrize("M,N,K", [(1, 384, 384), (255, 1152, 384), (257, 1536, 384),
                                   (4097, 1152, 384), (3001, 256, 64), (1000, 4096, 128),
                                   (20011, 1536, 384), (700, 2304, 192)])
@pytest.mark.parametrize("epi", [0, 1])
def test_gemm_weight_resident(ec, monkeypatch, M, N, K, epi):
    monkeypatch.setenv("EC_GEMM_WR", "1")
    g = torch.Generator(device="cuda").manual_seed(M * 5 + N + K + epi)
    A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    W = (0.05 * torch.randn(N, K, device="cuda", generator=g)).bfloat16()
    bias = torch.randn(N, device="cuda", generator=g)
    ref = A.float() @ W.float().t() + bias
    if epi == 1:
        ref = _gelu_as(ref)
    out = _gemm(ec, A, W, bias, None, epi, 0, N, torch.bfloat16).float()
    err = (out - ref).abs().max().item() / max(ref.abs().max().item(), 1e-6)
    assert err < 1e-2, f"rel err {err}"
    monkeypatch.setenv("EC_NO_GEMM_WR", "1")
    out2 = _gemm(ec, A, W, bias, None, epi, 0, N, torch.bfloat16).float()
    err2 = (out - out2).abs().max().item() / max(ref.abs().max().item(), 1e-6)
    assert err2 < 1e-2, f"weight-resident vs streaming rel diff {err2}"


@pytest.mark.parametrize("M,F", [(1, 3072), (300, 3072), (1029, 1536)])
@pytest.mark.parametrize("pair", [0, 1])
def test_gemm_swiglu(ec, monkeypatch, M, F, pair):
    if pair:
        monkeypatch.setenv("EC_GEMM_PAIR", "1")
    K = 1024
    g = torch.Generator(device="cuda").manual_seed(M + F)
    A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    Wg = (0.03 * torch.randn(F, K, device="cuda", generator=g)).bfloat16()
    Wu = (0.03 * torch.randn(F, K, device="cuda", generator=g)).bfloat16()
    # block-interleave 128 rows of gate, 128 rows of up (256-wide tiles)
    W = torch.stack([Wg.view(F // 128, 128, K), Wu.view(F // 128, 128, K)], 1).reshape(2 * F, K)
    out = _gemm(ec, A, W.contiguous(), None, None, 3, 0 if pair else 256, F, torch.bfloat16).float()
    gg = A.float() @ Wg.float().t()
    uu = A.float() @ Wu.float().t()
    ref = gg / (1 + torch.exp(-gg)) * uu
    err = (out - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1e-2, err


def _attn_ref(qkv, lens, heads, kv_heads, hd, q_off, k_off, v_off, causal):
    outs = []
    o = 0
    group = heads // kv_heads
    for L in lens:
        x = qkv[o:o + L].float()
        q = x[:, q_off:q_off + heads * hd].view(L, heads, hd).transpose(0, 1)
        k = x[:, k_off:k_off + kv_heads * hd].view(L, kv_heads, hd).transpose(0, 1)
        v = x[:, v_off:v_off + kv_heads * hd].view(L, kv_heads, hd).transpose(0, 1)
        k = k.repeat_interleave(group, 0)
        v = v.repeat_interleave(group, 0)
        s = q @ k.transpose(1, 2) / math.sqrt(hd)
        if causal:
            s = s.masked_fill(torch.triu(torch.ones(L, L, device=s.device, dtype=torch.bool), 1),
                              float("-inf"))
        p = torch.softmax(s, -1)
        outs.append((p @ v).transpose(0, 1).reshape(L, heads * hd))
        o += L
    return torch.cat(outs)


def _run_attention(ec, lens, hd, heads, kv, causal, key_boost=1.0, tol=2e-2):
    T = sum(lens)
    ld = (heads + 2 * kv) * hd
    g = torch.Generator(device="cuda").manual_seed(hd + heads)
    qkv = torch.randn(T, ld, device="cuda", generator=g)
    if key_boost != 1.0:
        # keys from position 128 on scaled up: the running row max jumps by
        # different amounts on different rows of the second key block
        o = 0
        for L in lens:
            qkv[o + 128:o + L, heads * hd:(heads + kv) * hd] *= key_boost
            o += L
    qkv = qkv.bfloat16()
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device="cuda")
    out = torch.zeros(T, heads * hd, dtype=torch.bfloat16, device="cuda")
    lens_h = np.asarray(lens, np.int32)
    torch.cuda.synchronize()
    import ctypes as C
    ec.check(ec.lib().ecdbg_attention(qkv.data_ptr(), ld, 0, heads * hd, (heads + kv) * hd,
                                      out.data_ptr(), C.c_void_p(cu.data_ptr()),
                                      lens_h.ctypes.data_as(C.POINTER(C.c_int32)), len(lens),
                                      heads, kv, hd, causal), "attention")
    ref = _attn_ref(qkv, lens, heads, kv, hd, 0, heads * hd, (heads + kv) * hd, causal)
    err = (out.float() - ref).abs().max().item()
    assert err < tol, err


# mixed lengths: sequences above 256 tokens run on the tcgen05 kernel, the
# others (head dims 32 / 64) on the short-sequence kernel
@pytest.mark.parametrize("hd,heads,kv,causal", [(32, 12, 12, 0), (64, 12, 12, 0), (128, 16, 8, 1),
                                                 (128, 4, 4, 0), (64, 2, 1, 1), (32, 4, 2, 1)])
def test_attention(ec, hd, heads, kv, causal):
    _run_attention(ec, [1, 5, 63, 64, 65, 200, 513, 17], hd, heads, kv, causal)


# rows whose running max grows past the lazy-rescale threshold next to rows
# whose max does not (the O rescale in TMEM is warp-collective)
@pytest.mark.parametrize("hd,heads,kv,causal", [(128, 4, 1, 0), (128, 16, 8, 1), (64, 12, 12, 0)])
def test_attention_rescale_mixed_rows(ec, hd, heads, kv, causal):
    _run_attention(ec, [300, 129, 513, 40], hd, heads, kv, causal, key_boost=3.0, tol=4e-2)


# the short kernel's fp16 probabilities with large, uneven logits: keys from
# position 128 on scaled by 4 (scores up to ~30 in log2 units, probabilities
# down to f16 underflow) next to sequences that never reach them
@pytest.mark.parametrize("hd,causal,tc", [(32, 0, 0), (64, 0, 0), (32, 1, 0), (32, 0, 1)])
def test_attention_short_large_logits(ec, monkeypatch, hd, causal, tc):
    if tc:
        monkeypatch.setenv("EC_SHORT_ATTN_TC", "1")
    _run_attention(ec, [256, 200, 129, 40, 130], hd, 4, 4 if not causal else 2, causal,
                   key_boost=4.0, tol=4e-2)


# only short sequences (1..256 tokens, edges included), on the short kernel
# (fp16 probabilities by default, bf16 with EC_SHORT_ATTN_BF16) and
# (EC_NO_SHORT_ATTN) on the tcgen05 kernel
@pytest.mark.parametrize("hd,heads,kv,causal,tc", [(32, 12, 12, 0, 0), (32, 4, 2, 1, 0),
                                                    (64, 12, 12, 0, 0), (64, 4, 2, 1, 0),
                                                    (64, 12, 12, 0, 1), (32, 12, 12, 0, 1),
                                                    (32, 12, 12, 0, 2), (64, 4, 2, 1, 2),
                                                    (32, 12, 12, 0, 3), (32, 4, 2, 0, 3)])
def test_attention_short_sequences(ec, monkeypatch, hd, heads, kv, causal, tc):
    if tc == 1:
        monkeypatch.setenv("EC_NO_SHORT_ATTN", "1")
    elif tc == 2:
        monkeypatch.setenv("EC_SHORT_ATTN_BF16", "1")
    elif tc == 3:  # the tcgen05 short-sequence kernel (head dim 32, no mask)
        monkeypatch.setenv("EC_SHORT_ATTN_TC", "1")
    rng = np.random.default_rng(hd * 7 + heads)
    lens = [int(x) for x in rng.integers(1, 257, 40)] + [256, 255, 16, 1]
    _run_attention(ec, lens, hd, heads, kv, causal)


def _ln_ref(x, g, b):
    # bert::layernorm: (x - mean) / (sqrt(var) + 1e-12) * g + b
    m = x.mean(-1, keepdim=True)
    v = ((x - m) ** 2).mean(-1, keepdim=True)
    return (x - m) / (v.sqrt() + 1e-12) * g + b


# GEMM + residual + LayerNorm on CTA clusters: H 384 (2 CTAs), 768 (3), 1024 (4);
# ragged M, K = H and K = 4H, output aliasing the residual as the model runs it
@pytest.mark.parametrize("M,N,K,alias", [(1, 384, 384, False), (200, 384, 1536, True),
                                         (4097, 384, 384, True), (999, 768, 768, False),
                                         (3000, 768, 3072, True), (257, 1024, 1024, True)])
def test_gemm_layernorm(ec, M, N, K, alias):
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    W = (0.05 * torch.randn(N, K, device="cuda", generator=g)).bfloat16()
    bias = 0.1 * torch.randn(N, device="cuda", generator=g)
    resid = torch.randn(M, N, device="cuda", generator=g)
    lg = 1 + 0.1 * torch.randn(N, device="cuda", generator=g)
    lb = 0.1 * torch.randn(N, device="cuda", generator=g)
    ref = _ln_ref(A.float() @ W.float().t() + bias + resid, lg, lb)
    out32 = resid if alias else torch.empty(M, N, device="cuda")
    outb = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    torch.cuda.synchronize()
    ec.check(ec.lib().ecdbg_gemm_ln(A.data_ptr(), W.data_ptr(), M, N, K, bias.data_ptr(),
                                    resid.data_ptr(), lg.data_ptr(), lb.data_ptr(),
                                    out32.data_ptr(), outb.data_ptr()), "gemm_ln")
    err = (out32 - ref).abs().max().item()
    assert err < 1e-2, err
    assert (outb.float() - ref).abs().max().item() < 5e-2


# fused FFN on CTA pairs (256-row tiles): ragged M (a pair whose odd CTA has
# no rows, or one row), the fp32 residual stream with the fp32 row stored, and
# the bf16 residual (the input rows themselves) with the bf16 row only
@pytest.mark.parametrize("M,H,F", [(1, 384, 1536), (200, 384, 1536), (4097, 384, 1536),
                                   (300, 256, 512), (129, 128, 256)])
@pytest.mark.parametrize("res", ["f32", "bf16"])
def test_fused_mlp(ec, M, H, F, res):
    g = torch.Generator(device="cuda").manual_seed(M + H + F)
    A = torch.randn(M, H, device="cuda", generator=g).bfloat16()
    W1 = (0.05 * torch.randn(F, H, device="cuda", generator=g)).bfloat16()
    W2 = (0.03 * torch.randn(H, F, device="cuda", generator=g)).bfloat16()
    b1 = 0.1 * torch.randn(F, device="cuda", generator=g)
    b2 = 0.1 * torch.randn(H, device="cuda", generator=g)
    resid = torch.randn(M, H, device="cuda", generator=g)
    lg = 1 + 0.1 * torch.randn(H, device="cuda", generator=g)
    lb = 0.1 * torch.randn(H, device="cuda", generator=g)
    out32 = torch.empty(M, H, device="cuda")
    outb = torch.empty(M, H, device="cuda", dtype=torch.bfloat16)
    torch.cuda.synchronize()
    f32 = res == "f32"
    ec.check(ec.lib().ecdbg_mlp(A.data_ptr(), W1.data_ptr(), W2.data_ptr(), b1.data_ptr(),
                                b2.data_ptr(), resid.data_ptr() if f32 else None, lg.data_ptr(),
                                lb.data_ptr(), out32.data_ptr() if f32 else None, outb.data_ptr(),
                                M, H, F), "mlp")
    u = _gelu_as(A.float() @ W1.float().t() + b1)
    p = u.bfloat16().float()  # the intermediate is bf16 on chip
    y = p @ W2.float().t() + b2 + (resid if f32 else A.float())
    ref = _ln_ref(y, lg, lb)
    if f32:
        err = (out32 - ref).abs().max().item()
        assert err < 2e-2, err
    assert (outb.float() - ref).abs().max().item() < 5e-2
