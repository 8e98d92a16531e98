"""Single-kernel parity on the GPU through the C ABI: the tcgen05 GEMM, varlen attention and
LayerNorm against fp32 references of the same op (torch on the device, numpy oracle on the host)."""

import numpy as np
import pytest

from oracle import modern_bert

pytestmark = pytest.mark.gpu


def _torch():
    import torch

    return torch


def _stream():
    return _torch().cuda.current_stream().cuda_stream


@pytest.mark.parametrize("act", ["bf16", "f16"])
@pytest.mark.parametrize("M,N,K,bn", [(1, 256, 64, 256), (127, 256, 768, 256), (128, 768, 768, 256),
                                      (1000, 2304, 768, 256), (4096, 768, 1152, 256), (300, 1152, 384, 128),
                                      (513, 384, 1536, 128), (20000, 768, 768, 256),
                                      # bn=512: two-CTA 256 x 256 tiles (tcgen05.mma.cta_group::2)
                                      (1, 256, 64, 512), (255, 768, 768, 512), (257, 2304, 768, 512),
                                      (4096, 768, 1152, 512), (20000, 2304, 768, 512)])
def test_gemm_matches_fp32(cuda_device, act, M, N, K, bn):
    torch = _torch()
    from ripvec_b200 import _lib as L

    dt = torch.bfloat16 if act == "bf16" else torch.float16
    code = L.RV_DTYPE_BF16 if act == "bf16" else L.RV_DTYPE_F16
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N)
    a = torch.randn(M, K, device="cuda", generator=g).to(dt)
    b = torch.randn(N, K, device="cuda", generator=g).to(dt)
    ref = a.float() @ b.float().T
    c32 = torch.empty(M, N, device="cuda", dtype=torch.float32)
    assert L.lib().rv_op_gemm(code, a.data_ptr(), b.data_ptr(), c32.data_ptr(), L.RV_DTYPE_F32, M, N, K, bn,
                              _stream()) == 0
    # f32 accumulation of exact products: differences come only from the summation order.
    tol = 1e-5 * K ** 0.5 * ref.abs().max().item() + 1e-3
    assert (c32 - ref).abs().max().item() < tol
    c16 = torch.empty(M, N, device="cuda", dtype=dt)
    assert L.lib().rv_op_gemm(code, a.data_ptr(), b.data_ptr(), c16.data_ptr(), code, M, N, K, bn, _stream()) == 0
    rel = ((c16.float() - ref).abs() / (ref.abs() + 1)).max().item()
    assert rel < (8e-3 if act == "bf16" else 1e-3)


def test_gemm_rejects_bad_shapes(cuda_device):
    from ripvec_b200 import _lib as L

    assert L.lib().rv_op_gemm(L.RV_DTYPE_BF16, 0, 0, 0, L.RV_DTYPE_F32, 128, 256, 100, 256, None) == L.RV_E_INVALID
    assert L.lib().rv_op_gemm(L.RV_DTYPE_BF16, 0, 0, 0, L.RV_DTYPE_F32, 128, 200, 128, 256, None) == L.RV_E_INVALID


def _attention_ref(qkv: np.ndarray, cu, heads, hd, window_half):
    H = heads * hd
    out = np.zeros((qkv.shape[0], H), np.float32)
    for b in range(len(cu) - 1):
        s0, s1 = cu[b], cu[b + 1]
        if s1 == s0:
            continue
        x = qkv[s0:s1]
        q = x[:, :H].reshape(-1, heads, hd)
        k = x[:, H:2 * H].reshape(-1, heads, hd)
        v = x[:, 2 * H:].reshape(-1, heads, hd)
        out[s0:s1] = modern_bert._attention(q, k, v, 1.0 / np.sqrt(hd), window_half, np.float32)
    return out


@pytest.mark.parametrize("impl", ["tc", "tc_poly", "mma"])
@pytest.mark.parametrize("act", ["bf16", "f16"])
@pytest.mark.parametrize("hd,heads,window", [(64, 12, -1), (64, 12, 64), (32, 12, -1), (64, 4, 64)])
def test_attention_matches_oracle(cuda_device, monkeypatch, impl, act, hd, heads, window):
    """head_dim 64 runs the tcgen05 kernel ("tc"; "tc_poly" with a quarter of the softmax
    exponentials on the FMA pipe, RV_ATTN_EXP2_POLY=1) or, with RV_ATTN_TC=0, the mma.sync
    kernel; at this op level head_dim 32 has only the mma.sync kernel."""
    torch = _torch()
    from ripvec_b200 import _lib as L

    if impl != "mma" and hd != 64:
        pytest.skip("the tcgen05 kernel covers head_dim 64")
    monkeypatch.setenv("RV_ATTN_TC", "0" if impl == "mma" else "1")
    monkeypatch.setenv("RV_ATTN_EXP2_POLY", "1" if impl == "tc_poly" else "0")

    lengths = [1, 17, 63, 64, 65, 129, 300, 512, 0, 700]
    cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    T = int(cu[-1])
    rng = np.random.default_rng(hd + heads + window)
    dt = torch.bfloat16 if act == "bf16" else torch.float16
    qkv = torch.from_numpy(rng.standard_normal((T, 3 * heads * hd)).astype(np.float32) * 1.5).to(dt).cuda()
    ctx = torch.zeros(T, heads * hd, device="cuda", dtype=dt)
    code = L.RV_DTYPE_BF16 if act == "bf16" else L.RV_DTYPE_F16
    rc = L.lib().rv_op_attention(code, qkv.data_ptr(), ctx.data_ptr(), cu.ctypes.data, len(lengths), heads, hd,
                                 window, float(1.0 / np.sqrt(hd)), _stream())
    assert rc == 0
    ref = _attention_ref(qkv.float().cpu().numpy(), cu, heads, hd, window)
    got = ctx.float().cpu().numpy()
    err = np.abs(got - ref).max()
    assert err < (3e-2 if act == "bf16" else 5e-3), err


@pytest.mark.parametrize("window", [-1, 64])
def test_attention_many_items_per_cta(cuda_device, monkeypatch, window):
    """Enough 128-query tiles that every persistent CTA of the tcgen05 kernel walks dozens of
    items, so Q, K/V and TMEM buffers rotate across item boundaries; ragged, empty and
    one-token sequences interleaved."""
    torch = _torch()
    from ripvec_b200 import _lib as L

    monkeypatch.setenv("RV_ATTN_TC", "1")
    heads, hd = 12, 64
    rng = np.random.default_rng(7 + window)
    lengths = rng.integers(64, 513, size=400)
    lengths[::37] = 0
    lengths[5::41] = 1
    cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    T = int(cu[-1])
    qkv = torch.from_numpy(rng.standard_normal((T, 3 * heads * hd)).astype(np.float32)).to(torch.bfloat16).cuda()
    ctx = torch.full((T, heads * hd), float("nan"), device="cuda", dtype=torch.bfloat16)
    rc = L.lib().rv_op_attention(L.RV_DTYPE_BF16, qkv.data_ptr(), ctx.data_ptr(), cu.ctypes.data, len(lengths),
                                 heads, hd, window, float(1.0 / np.sqrt(hd)), _stream())
    assert rc == 0
    ref = _attention_ref(qkv.float().cpu().numpy(), cu, heads, hd, window)
    got = ctx.float().cpu().numpy()
    assert np.isfinite(got).all(), "rows left unwritten"
    err = np.abs(got - ref).max()
    assert err < 3e-2, err


@pytest.mark.parametrize("hidden", [768, 384, 256])
def test_layernorm_matches_fp32(cuda_device, hidden):
    torch = _torch()
    from ripvec_b200 import _lib as L

    x = (torch.randn(3001, hidden, device="cuda") * 3 + 0.5).to(torch.bfloat16)
    gamma = torch.rand(hidden, device="cuda") + 0.5
    beta = torch.randn(hidden, device="cuda") * 0.1
    y = torch.empty_like(x)
    assert L.lib().rv_op_layernorm(L.RV_DTYPE_BF16, x.data_ptr(), y.data_ptr(), 3001, hidden, gamma.data_ptr(),
                                   beta.data_ptr(), 1e-5, _stream()) == 0
    ref = torch.nn.functional.layer_norm(x.float(), (hidden,), gamma, beta, 1e-5)
    assert (y.float() - ref).abs().max().item() < 3e-2


def test_exp2_poly_error_bound(cuda_device):
    """The FMA-pipe exponential of the tcgen05 softmax (rv_debug_exp2_poly) against the exact
    2^x (float64) and CUDA's exp2f (torch.exp2 on the device) over the softmax input range: relative
    error below 7.6e-5 on [-125, 126] (the polynomial's minimax error is 7.48e-5), and exactly 0
    below -125 and for masked (-inf) scores."""
    torch = _torch()
    from ripvec_b200 import _lib as L

    rng = np.random.default_rng(5)
    x = np.concatenate([np.linspace(-125.0, 126.0, 2_000_001), rng.uniform(-20.0, 8.0, 1_000_000),
                        np.arange(-125, 127, dtype=np.float64), np.arange(-125, 127) + 0.5,
                        [0.0, -0.0, 1e-30, -1e-30, 8.0]]).astype(np.float32)
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty_like(xd)
    assert L.lib().rv_debug_exp2_poly(xd.data_ptr(), yd.data_ptr(), x.size, _stream()) == L.RV_OK
    y = yd.cpu().numpy().astype(np.float64)
    exact = np.exp2(x.astype(np.float64))
    rel = np.abs(y - exact) / exact
    assert rel.max() < 7.6e-5, (rel.max(), x[np.argmax(rel)])
    cuda = torch.exp2(xd).cpu().numpy().astype(np.float64)
    assert (np.abs(y - cuda) / cuda).max() < 7.6e-5 + 2.0 ** -21

    low = np.array([-125.0001, -126.0, -200.0, -1e9, -np.inf], np.float32)
    ld = torch.from_numpy(low).cuda()
    lo = torch.full_like(ld, 1.0)
    assert L.lib().rv_debug_exp2_poly(ld.data_ptr(), lo.data_ptr(), low.size, _stream()) == L.RV_OK
    assert (lo.cpu().numpy() == 0.0).all()
